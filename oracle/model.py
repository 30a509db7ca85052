"""ORACLE (test infrastructure only) -- numpy restatement of the two-view model.

Computes in float64 so that it serves as the reference value the GPU path is
measured against.  Every function cites the reference code it restates:

  preprocess        backends/python/python_engine.py:176-188 (no resize when the
                    input already has the model resolution)
  patch_embed       backends/python/vit_encoder.py:123-167, croco_encoder.py:262-271
  positions         backends/python/rope2d.py:29-55   (y, x) row-major grid
  rope              backends/python/rope2d.py:65-146  base 100, half-split pairs,
                    first half of the rotary frequencies on y, second on x
  layer_norm        backends/python/vit_encoder.py:98-108 (eps 1e-6)
  gelu              backends/python/vit_encoder.py:18-20 (tanh approximation)
  encoder block     backends/python/croco_encoder.py:50-93, 142-168
  encoder           backends/python/croco_encoder.py:245-283
  decoder block     backends/python/croco_decoder.py:59-89, 146-184, 245-279
  decoder           backends/python/croco_decoder.py:395-434 (+ hook capture)
  24-d head         csrc/mps/mpsgraph_engine.mm:383-437, csrc/mps/graph_builder.hpp:267-322
                    (DPT: act_postprocess, layer_rn, bilinear fusion, head convs;
                    local features: MLP(enc || dec) -> pixel shuffle -> L2 norm)
  ref_simple head   backends/python/mast3r_model.py:86-156 with
                    backends/python/dpt_head.py:20-116 (the reference's own CPU head)
  retrieval         csrc/mps/mpsgraph_engine.mm:767-850, 1030-1117 (encoder output whitened,
                    L2 attention weights)

The 24-d head has no runnable reference here (Metal only), so its parity is pinned
only through the encoder/decoder fixtures; see the golden-vector script in
tests/golden/.
"""

from __future__ import annotations

import numpy as np

IMAGENET_MEAN = (0.485, 0.456, 0.406)
IMAGENET_STD = (0.229, 0.224, 0.225)


# ----------------------------------------------------------------------------- ops

def preprocess(img: np.ndarray) -> np.ndarray:
    """uint8 [H, W, 3] -> float [3, H, W]; python_engine.py:176-188 (float32 as there)."""
    x = img.astype(np.float32) / np.float32(255.0)
    x = (x - np.array(IMAGENET_MEAN, np.float32)) / np.array(IMAGENET_STD, np.float32)
    return np.transpose(x, (2, 0, 1)).astype(np.float64)


def layer_norm(x, w, b, eps=1e-6):
    """vit_encoder.py:98-108."""
    mu = x.mean(-1, keepdims=True)
    var = ((x - mu) ** 2).mean(-1, keepdims=True)
    return (x - mu) / np.sqrt(var + eps) * w + b


def gelu(x):
    """vit_encoder.py:18-20 (tanh approximation)."""
    return 0.5 * x * (1.0 + np.tanh(np.sqrt(2.0 / np.pi) * (x + 0.044715 * x ** 3)))


def linear(x, w, b=None):
    """vit_encoder.py:111-120: y = x W^T + b, W [out, in]."""
    y = x @ np.asarray(w).T
    return y if b is None else y + b


def softmax(x):
    m = x.max(-1, keepdims=True)
    e = np.exp(x - m)
    return e / e.sum(-1, keepdims=True)


def positions(hg: int, wg: int) -> np.ndarray:
    """rope2d.py:29-55: [N, 2] (y, x), row-major."""
    yy, xx = np.meshgrid(np.arange(hg), np.arange(wg), indexing="ij")
    return np.stack([yy.ravel(), xx.ravel()], -1)


def rope_tables(pos: np.ndarray, head_dim: int, base: float = 100.0):
    """cos/sin [N, head_dim/2] (rope2d.py:77-92, 118-131); angles in float32 as there."""
    nf = head_dim // 4
    freqs = (1.0 / (np.float32(base) ** (np.arange(nf, dtype=np.float32) / np.float32(nf)))).astype(np.float32)
    ay = pos[:, 0].astype(np.float32)[:, None] * freqs
    ax = pos[:, 1].astype(np.float32)[:, None] * freqs
    ang = np.concatenate([ay, ax], -1).astype(np.float32)
    return np.cos(ang).astype(np.float64), np.sin(ang).astype(np.float64)


def rope(t, cos, sin):
    """rope2d.py:133-146 on [h, N, dh]: pairs (i, i + dh/2)."""
    d2 = t.shape[-1] // 2
    t1, t2 = t[..., :d2], t[..., d2:]
    return np.concatenate([t1 * cos - t2 * sin, t1 * sin + t2 * cos], -1)


def attention(q, k, v, scale):
    """softmax(q k^T * scale) v on [h, N, dh]."""
    return softmax((q @ np.swapaxes(k, -1, -2)) * scale) @ v


def split_heads(x, h):
    n, d = x.shape
    return x.reshape(n, h, d // h).transpose(1, 0, 2)


def merge_heads(x):
    h, n, dh = x.shape
    return x.transpose(1, 0, 2).reshape(n, h * dh)


# ----------------------------------------------------------------------------- conv helpers (NHWC)

def conv2d(x, w, b=None, stride=1, pad=0):
    """NHWC conv, weight [out, in, kh, kw] (PyTorch layout)."""
    hh, ww, _ = x.shape
    co, ci, kh, kw = w.shape
    if pad:
        x = np.pad(x, ((pad, pad), (pad, pad), (0, 0)))
    ho = (hh + 2 * pad - kh) // stride + 1
    wo = (ww + 2 * pad - kw) // stride + 1
    wt = np.asarray(w).transpose(2, 3, 1, 0)  # [kh, kw, ci, co]
    out = np.zeros((ho, wo, co), np.result_type(x, wt))
    for dy in range(kh):
        for dx in range(kw):
            xs = x[dy: dy + stride * (ho - 1) + 1: stride, dx: dx + stride * (wo - 1) + 1: stride]
            out += xs @ wt[dy, dx]
    return out if b is None else out + b


def conv_transpose_k_eq_s(x, w, b, s):
    """ConvTranspose2d with kernel == stride, padding 0 (weight [in, out, s, s]):
    out[s*y + dy, s*x + dx, co] = b[co] + sum_ci x[y, x, ci] w[ci, co, dy, dx]."""
    hh, ww, ci = x.shape
    co = w.shape[1]
    y = np.einsum("yxc,codk->ydxko", x, np.asarray(w))  # [H, s, W, s, co]
    return y.reshape(hh * s, ww * s, co) + b


def resize_bilinear(x, ho, wo):
    """Bilinear, half-pixel centres, align_corners=False (graph_builder.hpp:292-297)."""
    hi, wi, _ = x.shape

    def axis(n_out, n_in):
        src = (np.arange(n_out) + 0.5) * (n_in / n_out) - 0.5
        src = np.maximum(src, 0.0)
        i0 = np.minimum(np.floor(src).astype(np.int64), n_in - 1)
        i1 = np.minimum(i0 + 1, n_in - 1)
        return i0, i1, src - i0

    y0, y1, fy = axis(ho, hi)
    x0, x1, fx = axis(wo, wi)
    fy = fy[:, None, None]
    fx = fx[None, :, None]
    top = x[y0][:, x0] * (1 - fx) + x[y0][:, x1] * fx
    bot = x[y1][:, x0] * (1 - fx) + x[y1][:, x1] * fx
    return top * (1 - fy) + bot * fy


def interpolate_bilinear_ref(x, ho, wo):
    """dpt_head.py:72-116 (src = i * H/H_out, no half-pixel offset), on NHWC."""
    hi, wi, _ = x.shape
    sh, sw = hi / ho, wi / wo
    ys = np.arange(ho) * sh
    xs = np.arange(wo) * sw
    h0 = ys.astype(np.int64)
    w0 = xs.astype(np.int64)
    h1 = np.minimum(h0 + 1, hi - 1)
    w1 = np.minimum(w0 + 1, wi - 1)
    fh = (ys - h0)[:, None, None]
    fw = (xs - w0)[None, :, None]
    return ((1 - fh) * (1 - fw) * x[h0][:, w0] + (1 - fh) * fw * x[h0][:, w1]
            + fh * (1 - fw) * x[h1][:, w0] + fh * fw * x[h1][:, w1])


# ----------------------------------------------------------------------------- model

class Model:
    """Restatement of encoder + decoder + heads for one image pair.

    ``dtype`` float64 (default) is the parity reference; float32 is the arithmetic the
    reference's numpy path starts from and is used to time the CPU baseline.
    """

    def __init__(self, weights: dict, dims, dtype=np.float64):
        self.dt = np.dtype(dtype)
        self.w = {k: np.asarray(v, self.dt) for k, v in weights.items()}
        self.d = dims

    # croco_encoder.py:245-283
    def encode(self, img_chw: np.ndarray):
        d, W = self.d, self.w
        p = d.patch
        _, hh, ww = img_chw.shape
        hg, wg = hh // p, ww // p
        img_chw = img_chw.astype(self.dt)
        patches = img_chw[:, : hg * p, : wg * p].reshape(3, hg, p, wg, p).transpose(1, 3, 0, 2, 4)
        x = patches.reshape(hg * wg, 3 * p * p) @ W["patch_embed.proj.weight"].reshape(d.enc_dim, -1).T
        x = x + W["patch_embed.proj.bias"]
        cos, sin = rope_tables(positions(hg, wg), d.head_dim)
        cos, sin = cos.astype(self.dt), sin.astype(self.dt)
        scale = d.head_dim ** -0.5
        for i in range(d.enc_depth):
            b = f"enc_blocks.{i}."
            h = layer_norm(x, W[b + "norm1.weight"], W[b + "norm1.bias"])
            qkv = linear(h, W[b + "attn.qkv.weight"], W[b + "attn.qkv.bias"])
            q, k, v = np.split(qkv, 3, -1)
            q = rope(split_heads(q, d.enc_heads), cos, sin)
            k = rope(split_heads(k, d.enc_heads), cos, sin)
            o = merge_heads(attention(q, k, split_heads(v, d.enc_heads), scale))
            x = x + linear(o, W[b + "attn.proj.weight"], W[b + "attn.proj.bias"])
            h = layer_norm(x, W[b + "norm2.weight"], W[b + "norm2.bias"])
            h = gelu(linear(h, W[b + "mlp.fc1.weight"], W[b + "mlp.fc1.bias"]))
            x = x + linear(h, W[b + "mlp.fc2.weight"], W[b + "mlp.fc2.bias"])
        x = layer_norm(x, W["enc_norm.weight"], W["enc_norm.bias"])
        return x, (hg, wg)

    # croco_decoder.py:245-279
    def _dec_block(self, pre, x, y, cos_x, sin_x, cos_y, sin_y):
        d, W = self.d, self.w
        hd = d.dec_heads
        scale = d.head_dim ** -0.5
        h = layer_norm(x, W[pre + "norm1.weight"], W[pre + "norm1.bias"])
        qkv = linear(h, W[pre + "attn.qkv.weight"], W[pre + "attn.qkv.bias"])
        q, k, v = np.split(qkv, 3, -1)
        q = rope(split_heads(q, hd), cos_x, sin_x)
        k = rope(split_heads(k, hd), cos_x, sin_x)
        o = merge_heads(attention(q, k, split_heads(v, hd), scale))
        x = x + linear(o, W[pre + "attn.proj.weight"], W[pre + "attn.proj.bias"])
        h = layer_norm(x, W[pre + "norm2.weight"], W[pre + "norm2.bias"])
        yn = layer_norm(y, W[pre + "norm_y.weight"], W[pre + "norm_y.bias"])
        q = rope(split_heads(linear(h, W[pre + "cross_attn.projq.weight"], W[pre + "cross_attn.projq.bias"]), hd),
                 cos_x, sin_x)
        k = rope(split_heads(linear(yn, W[pre + "cross_attn.projk.weight"], W[pre + "cross_attn.projk.bias"]), hd),
                 cos_y, sin_y)
        v = split_heads(linear(yn, W[pre + "cross_attn.projv.weight"], W[pre + "cross_attn.projv.bias"]), hd)
        o = merge_heads(attention(q, k, v, scale))
        x = x + linear(o, W[pre + "cross_attn.proj.weight"], W[pre + "cross_attn.proj.bias"])
        h = layer_norm(x, W[pre + "norm3.weight"], W[pre + "norm3.bias"])
        h = gelu(linear(h, W[pre + "mlp.fc1.weight"], W[pre + "mlp.fc1.bias"]))
        return x + linear(h, W[pre + "mlp.fc2.weight"], W[pre + "mlp.fc2.bias"])

    # croco_decoder.py:395-434, with the DPT hooks of mpsgraph_engine.mm:320-369
    def decode(self, enc1, enc2, grid):
        d, W = self.d, self.w
        cos, sin = rope_tables(positions(*grid), d.head_dim)
        cos, sin = cos.astype(self.dt), sin.astype(self.dt)
        p1 = linear(enc1, W["decoder_embed.weight"], W["decoder_embed.bias"])
        p2 = linear(enc2, W["decoder_embed.weight"], W["decoder_embed.bias"])
        outs = []
        for pre, x, y in (("dec_blocks", p1, p2), ("dec_blocks2", p2, p1)):
            hooks = []
            for i in range(d.dec_depth):
                x = self._dec_block(f"{pre}.{i}.", x, y, cos, sin, cos, sin)
                if i in d.hooks[:2]:
                    hooks.append(x)
            x = layer_norm(x, W["dec_norm.weight"], W["dec_norm.bias"])
            hooks.append(x)
            outs.append((x, hooks))
        return outs

    # mpsgraph_engine.mm:383-422 + graph_builder.hpp:267-299
    def dpt(self, head: str, enc, hooks, grid, out_hw):
        d, W = self.d, self.w
        hg, wg = grid
        t = head + ".dpt."

        def conv1x1(x, key):
            return linear(x, W[t + key + ".weight"][:, :, 0, 0], W[t + key + ".bias"])

        h0 = enc.reshape(hg, wg, -1)
        h1, h2, h3 = (h.reshape(hg, wg, -1) for h in hooks)
        f0 = conv_transpose_k_eq_s(conv1x1(h0, "act_postprocess.0.0"), W[t + "act_postprocess.0.1.weight"],
                                   W[t + "act_postprocess.0.1.bias"], 4)
        f1 = conv_transpose_k_eq_s(conv1x1(h1, "act_postprocess.1.0"), W[t + "act_postprocess.1.1.weight"],
                                   W[t + "act_postprocess.1.1.bias"], 2)
        f2 = conv1x1(h2, "act_postprocess.2.0")
        f3 = conv2d(conv1x1(h3, "act_postprocess.3.0"), W[t + "act_postprocess.3.1.weight"],
                    W[t + "act_postprocess.3.1.bias"], stride=2, pad=1)
        f = [conv2d(fk, W[t + f"scratch.layer_rn.{k}.weight"], None, 1, 1) for k, fk in enumerate((f0, f1, f2, f3))]
        H0, W0 = f[0].shape[:2]
        fused = f[0] + resize_bilinear(f[1], H0, W0) + resize_bilinear(f[2], H0, W0) + resize_bilinear(f[3], H0, W0)
        x = resize_bilinear(fused, 2 * H0, 2 * W0)
        x = np.maximum(conv2d(x, W[t + "head.0.weight"], W[t + "head.0.bias"], 1, 1), 0)
        x = resize_bilinear(x, 4 * H0, 4 * W0)
        x = np.maximum(conv2d(x, W[t + "head.2.weight"], W[t + "head.2.bias"], 1, 1), 0)
        x = linear(x, W[t + "head.4.weight"][:, :, 0, 0], W[t + "head.4.bias"])
        if x.shape[:2] != tuple(out_hw):
            x = resize_bilinear(x, *out_hw)
        return x[..., :3], x[..., 3]

    # mpsgraph_engine.mm:425-437 + graph_builder.hpp:300-322
    def local_features(self, head: str, enc, dec, grid):
        d, W = self.d, self.w
        f = head + ".head_local_features."
        x = np.concatenate([enc, dec], -1)
        x = gelu(linear(x, W[f + "fc1.weight"], W[f + "fc1.bias"]))
        x = linear(x, W[f + "fc2.weight"], W[f + "fc2.bias"])
        hg, wg = grid
        p = d.patch
        x = x.reshape(hg, wg, p, p, d.desc_dim + 1).transpose(0, 2, 1, 3, 4).reshape(hg * p, wg * p, -1)
        desc = x[..., : d.desc_dim]
        return desc / np.sqrt((desc ** 2).sum(-1, keepdims=True) + 1e-8)

    # mast3r_model.py:86-156 (the reference's own CPU head; 256-d raw descriptors)
    def ref_simple_head(self, head: str, enc, dec, grid, out_hw):
        W = self.w
        hg, wg = grid
        t = head + ".dpt."
        f = head + ".head_local_features."
        comb = np.concatenate([dec, enc], -1)
        raw = linear(gelu(linear(comb, W[f + "fc1.weight"], W[f + "fc1.bias"])), W[f + "fc2.weight"],
                     W[f + "fc2.bias"])
        sp = dec.reshape(hg, wg, -1)
        c = sp.shape[-1]
        feat = sp[..., :256] if c >= 256 else np.tile(sp, (1, 1, 256 // c + 1))[..., :256]
        x = np.maximum(conv2d(feat, W[t + "head.0.weight"], W[t + "head.0.bias"], 1, 1), 0)
        x = np.maximum(conv2d(x, W[t + "head.2.weight"], W[t + "head.2.bias"], 1, 1), 0)
        x = conv2d(x, W[t + "head.4.weight"], W[t + "head.4.bias"], 1, 0)
        x = interpolate_bilinear_ref(x, *out_hw)
        desc = interpolate_bilinear_ref(raw[:, :256].reshape(hg, wg, 256), *out_hw)
        return x[..., :3], desc, x[..., 3]

    def retrieval(self, img: np.ndarray, m: np.ndarray, p: np.ndarray):
        """Retrieval features of one image (csrc/mps/mpsgraph_engine.mm:767-850, encode_retrieval
        :1030-1117): the encoder output x [N, D] (after enc_norm) whitened as (x - m) @ P, and
        the per-token weights ||w||^2 / (sum over tokens of ||w||^2 + 1e-8).  No runnable
        reference exists for this (Metal only): restated from the graph source."""
        x, _ = self.encode(preprocess(img))
        w = (x - np.asarray(m, self.dt).reshape(1, -1)) @ np.asarray(p, self.dt)
        sq = (w * w).sum(-1)
        return w, sq / (sq.sum() + 1e-8)

    def forward(self, img1: np.ndarray, img2: np.ndarray, head: str = "mast3r24"):
        """Full pair: uint8 [H, W, 3] x2 -> dict of pts3d/conf/desc per view (float64)."""
        hh, ww = img1.shape[:2]
        e1, grid = self.encode(preprocess(img1))
        e2, _ = self.encode(preprocess(img2))
        (d1, hk1), (d2, hk2) = self.decode(e1, e2, grid)
        out = {"enc_1": e1, "enc_2": e2, "dec_1": d1, "dec_2": d2}
        for v, (e, dd, hk) in enumerate(((e1, d1, hk1), (e2, d2, hk2)), 1):
            name = f"downstream_head{v}"
            if head == "ref_simple":
                pts, desc, conf = self.ref_simple_head(name, e, dd, grid, (hh, ww))
            else:
                pts, conf = self.dpt(name, e, hk, grid, (hh, ww))
                desc = self.local_features(name, e, dd, grid)
            out[f"pts3d_{v}"] = pts
            out[f"conf_{v}"] = conf
            out[f"desc_{v}"] = desc
        return out
