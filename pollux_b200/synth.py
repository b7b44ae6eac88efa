"""Seeded synthetic workloads with the shapes and value distributions of the
benchmark configurations (no dataset or checkpoint is involved).

* config 1 -- one 1152x1152 fp32 weight, N(0, 0.02^2), seed 0.
* config 2 -- Pollux-1152-like backbone: 12 layers of QKV [3456,1152],
  O [1152,1152], up [4608,1152], down [1152,4608], fp32 N(0, 0.02^2), seed 1.
* config 3 -- Pollux-1920-like backbone: 18 layers of [5760,1920], [1920,1920],
  [7680,1920], [1920,7680], bf16 N(0, 0.02^2), seed 2.
* config 4 -- stress atoms, seed 3: 40 % scaled codewords plus noise, 20 % near
  the origin, 20 % midpoints of codeword pairs, 20 % isotropic N(0, 1).
* config 5 -- packed indices of a [7680,1920] layer, uniform in [0, 196560],
  fp16 row scales uniform in [0.01, 0.1].

Weight shapes follow nn.Linear ([out_features, in_features]); atoms run along
in_features (pack.py:161, pollux.py:495).
"""
from __future__ import annotations

import torch

H24_DIM = 24
H24_KISSING_COUNT = 196_560

CONFIG2_LAYER_SHAPES = [(3456, 1152), (1152, 1152), (4608, 1152), (1152, 4608)]
CONFIG2_LAYERS = 12
CONFIG3_LAYER_SHAPES = [(5760, 1920), (1920, 1920), (7680, 1920), (1920, 7680)]
CONFIG3_LAYERS = 18
CONFIG5_SHAPE = (7680, 1920)


def _gen(seed: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(int(seed))
    return g


def config1_weight(device="cpu") -> torch.Tensor:
    """[1152, 1152] fp32 N(0, 0.02^2) from seed 0 (CPU generator, then moved)."""
    g = _gen(0, "cpu")
    return (torch.randn(1152, 1152, generator=g) * 0.02).to(device)


def backbone_shapes(config: int) -> list[tuple[int, int]]:
    if config == 2:
        return CONFIG2_LAYER_SHAPES * CONFIG2_LAYERS
    if config == 3:
        return CONFIG3_LAYER_SHAPES * CONFIG3_LAYERS
    raise ValueError(f"no backbone for config {config}")


def backbone_weights(config: int, device="cuda", seed: int | None = None,
                     shapes: list[tuple[int, int]] | None = None) -> list[torch.Tensor]:
    """All weight matrices of config 2 (fp32) or config 3 (bf16), N(0, 0.02^2)."""
    if seed is None:
        seed = 1 if config == 2 else 2
    dtype = torch.float32 if config == 2 else torch.bfloat16
    g = _gen(seed, device)
    out = []
    for (o, i) in (shapes if shapes is not None else backbone_shapes(config)):
        w = torch.randn(o, i, generator=g, device=device, dtype=torch.float32) * 0.02
        out.append(w.to(dtype))
    return out


STRESS_CATEGORIES = ("codeword", "near_origin", "midpoint", "isotropic")


def stress_atoms(n: int, codebook_f32: torch.Tensor, seed: int = 3, device="cpu",
                 return_category: bool = False):
    """[n, 24] fp32 config-4 atoms.  ``codebook_f32`` is the [196561, 24] table.
    With return_category, also the category of each atom (an index into
    STRESS_CATEGORIES)."""
    g = _gen(seed, device)
    cb = codebook_f32.to(device=device, dtype=torch.float32)
    cat = torch.randint(0, 10, (n,), generator=g, device=device)
    i1 = torch.randint(1, H24_KISSING_COUNT + 1, (n,), generator=g, device=device)
    i2 = torch.randint(1, H24_KISSING_COUNT + 1, (n,), generator=g, device=device)
    scale = torch.rand(n, 1, generator=g, device=device) * 1.5 + 0.5
    noise = torch.randn(n, H24_DIM, generator=g, device=device) * 0.05
    iso = torch.randn(n, H24_DIM, generator=g, device=device)
    d = torch.randn(n, H24_DIM, generator=g, device=device)
    d = d / d.norm(dim=1, keepdim=True).clamp_min(1e-12)
    r = torch.rand(n, 1, generator=g, device=device) * 0.6
    near_codeword = cb[i1] * scale + noise
    near_origin = d * r
    midpoint = (cb[i1] + cb[i2]) * 0.5
    out = torch.where((cat < 4)[:, None], near_codeword,
          torch.where((cat < 6)[:, None], near_origin,
          torch.where((cat < 8)[:, None], midpoint, iso))).contiguous()
    if return_category:
        category = torch.where(cat < 4, 0, torch.where(cat < 6, 1, torch.where(cat < 8, 2, 3)))
        return out, category
    return out


def config5_layer(seed: int = 5, device="cuda", shape=CONFIG5_SHAPE):
    """(indices int32 [rows*in/24], sigma16 fp16 [rows]) of one config-5 layer."""
    rows, in_f = shape
    g = _gen(seed, device)
    n = rows * in_f // H24_DIM
    idx = torch.randint(0, H24_KISSING_COUNT + 1, (n,), generator=g, device=device,
                        dtype=torch.int64).to(torch.int32)
    sigma = (torch.rand(rows, generator=g, device=device) * 0.09 + 0.01).to(torch.float16)
    return idx, sigma
