"""Model dimensions and seeded random-init weights in the reference's CroCo key layout.

The reference checkpoints are not available offline, so weights are generated from a
seed: truncated normal (std 0.02, resampled beyond +-2 std) for every weight matrix,
biases 0, LayerNorm gamma 1 / beta 0 -- or, with ``randomize_affine=True`` (used by
the parity tests so that every bias and LayerNorm parameter is exercised), small
random biases and LayerNorm parameters as well.

Key layout follows the reference loaders:
  encoder   mast3r_runtime/backends/python/croco_encoder.py:196-239
  decoder   mast3r_runtime/backends/python/croco_decoder.py:308-388
  heads     csrc/mps/mpsgraph_engine.mm:177-222 (DPT + local features)
Dimensions follow csrc/mps/graph_builder.hpp:67-77 and csrc/common/types.hpp:51-69.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from pathlib import Path

import numpy as np


@dataclass(frozen=True)
class ModelDims:
    """Architecture of one model variant (encoder, decoder, heads)."""

    name: str
    patch: int
    enc_dim: int
    enc_depth: int
    enc_heads: int
    enc_mlp: int
    dec_dim: int = 768
    dec_depth: int = 12
    dec_heads: int = 12
    dec_mlp: int = 3072
    lf_hidden: int = 4096
    desc_dim: int = 24
    head_dim: int = 64
    dpt_dims: tuple = (96, 192, 384, 768)
    dpt_feat: int = 256
    dpt_head: int = 128

    @property
    def lf_in(self) -> int:
        return self.enc_dim + self.dec_dim

    @property
    def lf_out(self) -> int:
        return (self.desc_dim + 1) * self.patch * self.patch

    @property
    def hooks(self) -> tuple:
        """Decoder blocks whose outputs feed DPT levels 1..3 (mpsgraph_engine.mm:320-322)."""
        d = self.dec_depth
        return (d // 2 - 1, d * 3 // 4 - 1, d - 1)


# Variant table (mast3r_runtime/core/config.py:19-28 variant names).
VARIANTS: dict[str, ModelDims] = {
    "dune_vit_small_336": ModelDims("dune_vit_small_336", 14, 384, 12, 6, 1536),
    "dune_vit_small_448": ModelDims("dune_vit_small_448", 14, 384, 12, 6, 1536),
    "dune_vit_base_336": ModelDims("dune_vit_base_336", 14, 768, 12, 12, 3072),
    "dune_vit_base_448": ModelDims("dune_vit_base_448", 14, 768, 12, 12, 3072),
    "mast3r_vit_large": ModelDims("mast3r_vit_large", 16, 1024, 24, 16, 4096, lf_hidden=7168),
}


def tiny_dims(patch: int = 16, enc_dim: int = 128, enc_depth: int = 2, enc_heads: int = 2,
              dec_dim: int = 128, dec_depth: int = 4, dec_heads: int = 2, lf_hidden: int = 256) -> ModelDims:
    """A small model of the same architecture, for golden fixtures and fast tests."""
    return ModelDims("tiny", patch, enc_dim, enc_depth, enc_heads, 4 * enc_dim,
                     dec_dim=dec_dim, dec_depth=dec_depth, dec_heads=dec_heads, dec_mlp=4 * dec_dim,
                     lf_hidden=lf_hidden)


def _trunc_normal(rng: np.random.Generator, shape, std: float) -> np.ndarray:
    x = rng.standard_normal(shape, dtype=np.float32).reshape(-1)
    bad = np.flatnonzero(np.abs(x) > 2.0)
    while bad.size:  # resample only the rejected entries
        x[bad] = rng.standard_normal(bad.size, dtype=np.float32)
        bad = bad[np.abs(x[bad]) > 2.0]
    return (x * np.float32(std)).reshape(shape)


def round_to_16bit(x: np.ndarray, dtype: str) -> np.ndarray:
    """float32 values rounded (to nearest even) to the nearest fp16 / bf16 value, kept as
    float32 (exactly representable in the 16-bit type)."""
    x = np.ascontiguousarray(x, np.float32)
    if dtype == "fp16":
        return x.astype(np.float16).astype(np.float32)
    if dtype == "bf16":
        u = x.view(np.uint32).astype(np.uint64)
        r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
        return r.astype(np.uint32).view(np.float32)
    raise ValueError(f"unknown 16-bit type {dtype!r}")


def weight_shapes(d: ModelDims) -> dict[str, tuple]:
    """Every tensor of a unified checkpoint, in a fixed order."""
    s: dict[str, tuple] = {}
    e, p = d.enc_dim, d.patch
    s["patch_embed.proj.weight"] = (e, 3, p, p)
    s["patch_embed.proj.bias"] = (e,)
    for i in range(d.enc_depth):
        b = f"enc_blocks.{i}."
        s[b + "norm1.weight"] = (e,)
        s[b + "norm1.bias"] = (e,)
        s[b + "attn.qkv.weight"] = (3 * e, e)
        s[b + "attn.qkv.bias"] = (3 * e,)
        s[b + "attn.proj.weight"] = (e, e)
        s[b + "attn.proj.bias"] = (e,)
        s[b + "norm2.weight"] = (e,)
        s[b + "norm2.bias"] = (e,)
        s[b + "mlp.fc1.weight"] = (d.enc_mlp, e)
        s[b + "mlp.fc1.bias"] = (d.enc_mlp,)
        s[b + "mlp.fc2.weight"] = (e, d.enc_mlp)
        s[b + "mlp.fc2.bias"] = (e,)
    s["enc_norm.weight"] = (e,)
    s["enc_norm.bias"] = (e,)
    c = d.dec_dim
    s["decoder_embed.weight"] = (c, e)
    s["decoder_embed.bias"] = (c,)
    s["mask_token"] = (1, 1, c)
    for pre in ("dec_blocks", "dec_blocks2"):
        for i in range(d.dec_depth):
            b = f"{pre}.{i}."
            for n in ("norm1", "norm2", "norm_y", "norm3"):
                s[b + n + ".weight"] = (c,)
                s[b + n + ".bias"] = (c,)
            s[b + "attn.qkv.weight"] = (3 * c, c)
            s[b + "attn.qkv.bias"] = (3 * c,)
            s[b + "attn.proj.weight"] = (c, c)
            s[b + "attn.proj.bias"] = (c,)
            for n in ("projq", "projk", "projv", "proj"):
                s[b + f"cross_attn.{n}.weight"] = (c, c)
                s[b + f"cross_attn.{n}.bias"] = (c,)
            s[b + "mlp.fc1.weight"] = (d.dec_mlp, c)
            s[b + "mlp.fc1.bias"] = (d.dec_mlp,)
            s[b + "mlp.fc2.weight"] = (c, d.dec_mlp)
            s[b + "mlp.fc2.bias"] = (c,)
    s["dec_norm.weight"] = (c,)
    s["dec_norm.bias"] = (c,)
    c0, c1, c2, c3 = d.dpt_dims
    for h in ("downstream_head1", "downstream_head2"):
        t = h + ".dpt."
        s[t + "act_postprocess.0.0.weight"] = (c0, e, 1, 1)
        s[t + "act_postprocess.0.0.bias"] = (c0,)
        s[t + "act_postprocess.0.1.weight"] = (c0, c0, 4, 4)   # ConvTranspose2d [in, out, kh, kw]
        s[t + "act_postprocess.0.1.bias"] = (c0,)
        s[t + "act_postprocess.1.0.weight"] = (c1, c, 1, 1)
        s[t + "act_postprocess.1.0.bias"] = (c1,)
        s[t + "act_postprocess.1.1.weight"] = (c1, c1, 2, 2)   # ConvTranspose2d [in, out, kh, kw]
        s[t + "act_postprocess.1.1.bias"] = (c1,)
        s[t + "act_postprocess.2.0.weight"] = (c2, c, 1, 1)
        s[t + "act_postprocess.2.0.bias"] = (c2,)
        s[t + "act_postprocess.3.0.weight"] = (c3, c, 1, 1)
        s[t + "act_postprocess.3.0.bias"] = (c3,)
        s[t + "act_postprocess.3.1.weight"] = (c3, c3, 3, 3)   # Conv2d stride 2 pad 1
        s[t + "act_postprocess.3.1.bias"] = (c3,)
        for k, ck in enumerate(d.dpt_dims):
            s[t + f"scratch.layer_rn.{k}.weight"] = (d.dpt_feat, ck, 3, 3)
        s[t + "head.0.weight"] = (d.dpt_head, d.dpt_feat, 3, 3)
        s[t + "head.0.bias"] = (d.dpt_head,)
        s[t + "head.2.weight"] = (d.dpt_head, d.dpt_head, 3, 3)
        s[t + "head.2.bias"] = (d.dpt_head,)
        s[t + "head.4.weight"] = (4, d.dpt_head, 1, 1)
        s[t + "head.4.bias"] = (4,)
        f = h + ".head_local_features."
        s[f + "fc1.weight"] = (d.lf_hidden, d.lf_in)
        s[f + "fc1.bias"] = (d.lf_hidden,)
        s[f + "fc2.weight"] = (d.lf_out, d.lf_hidden)
        s[f + "fc2.bias"] = (d.lf_out,)
    return s


def make_weights(d: ModelDims, seed: int = 0, std: float = 0.02,
                 randomize_affine: bool = False, checkpoint_dtype: str | None = None) -> dict[str, np.ndarray]:
    """Seeded float32 weights for every tensor of ``weight_shapes(d)``.

    Weight matrices: truncated normal (std ``std``, +-2 std).  Biases: 0, LayerNorm
    gamma 1 / beta 0 -- unless ``randomize_affine``, in which case biases ~ N(0, std^2)
    and gamma ~ 1 + N(0, 0.1^2), beta ~ N(0, 0.05^2).

    ``checkpoint_dtype`` ("fp16" / "bf16"): a checkpoint stored in that 16-bit type --
    every value rounded to it (the reference's checkpoints are 16-bit; its CPU path
    upcasts them to float32), so a CPU model and a 16-bit GPU model read the same
    weight values.
    """
    rng = np.random.default_rng(seed)
    out: dict[str, np.ndarray] = {}
    for key, shape in weight_shapes(d).items():
        is_norm = ".norm" in key or key.startswith("enc_norm") or key.startswith("dec_norm")
        if key.endswith(".bias"):
            if randomize_affine:
                sd = 0.05 if is_norm else std
                out[key] = (rng.standard_normal(shape, dtype=np.float32) * np.float32(sd))
            else:
                out[key] = np.zeros(shape, np.float32)
        elif is_norm:
            if randomize_affine:
                out[key] = (1.0 + 0.1 * rng.standard_normal(shape, dtype=np.float32)).astype(np.float32)
            else:
                out[key] = np.ones(shape, np.float32)
        else:
            out[key] = _trunc_normal(rng, shape, std)
    if checkpoint_dtype is not None:
        out = {k: round_to_16bit(v, checkpoint_dtype) for k, v in out.items()}
    return out


def make_retrieval_weights(d: ModelDims, seed: int = 0) -> dict[str, np.ndarray]:
    """Seeded whitening weights of a retrieval checkpoint (the reference's
    retrieval.safetensors, csrc/mps/mpsgraph_engine.mm:770-787): prewhiten.m [enc_dim] (the
    feature mean) and prewhiten.p [enc_dim, enc_dim] (the whitening projection)."""
    rng = np.random.default_rng(seed)
    e = d.enc_dim
    return {"prewhiten.m": (0.1 * rng.standard_normal(e)).astype(np.float32),
            "prewhiten.p": (rng.standard_normal((e, e)) / np.sqrt(e)).astype(np.float32)}


def save_safetensors(path: str | Path, tensors: dict[str, np.ndarray]) -> Path:
    """Write ``tensors`` as an F32 safetensors file (the checkpoint format the loader reads)."""
    from safetensors.numpy import save_file

    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    save_file({k: np.ascontiguousarray(v, np.float32) for k, v in tensors.items()}, str(path))
    return path
