"""Drop-in mirror of the hot-path interface of the reference's ``castor.py``
(alavicka/pollux), backed by libh24.so on B200 (sm_100a).

Same names, signatures, argument meaning and error behaviour as the reference:

* constants ........................... castor.py:34-68
* get_h24_codebook ..................... castor.py:193-199
* centers_to_indices ................... castor.py:202-223
* pack_indices / unpack_indices ........ castor.py:226-260
* codebook_fingerprint ................. castor.py:263-266
* shape helpers ........................ castor.py:269-306
* row-RMS helpers ...................... castor.py:309-339
* castor_quantize_leech ................ castor.py:487-560
* CastorQuantizeLeech .................. castor.py:563-580
* project_h24_ / project_h24_many ...... the H24 block of pollux_step (pollux.py:874-884),
                                         fused and batched over parameters

Device policy: the work always runs on a CUDA device through libh24.  Tensors
on the host are staged through the current CUDA device and the result is
returned on the caller's device.  There is no CPU or Triton code path; without
a GPU or without the library every hot-path call raises.
"""
from __future__ import annotations

import ctypes
import math
from functools import lru_cache

import numpy as np
import torch

from . import _native as N

# ---------------------------------------------------------------------------
# Constants (castor.py:34-68)
# ---------------------------------------------------------------------------
friction_c: float = math.sqrt(2.0)
G24: float = 0.065771
gamma: float = G24
H24_DIM: int = 24
s_lattice: float = 1.0 / friction_c
NUMERICAL_EPSILON: float = 1e-8
H24_KISSING_COUNT = 196_560
H24_CODEBOOK_COUNT = H24_KISSING_COUNT + 1
H24_INDEX_BITS = 18
H24_INDEX_MASK = (1 << H24_INDEX_BITS) - 1
BACKBONE_BITS_PER_PARAM = 0.76
BITS_PER_PARAM_INDEX = 18 / H24_DIM
INDICES_PER_CHUNK = 4
BYTES_PER_CHUNK = 9
LEECH_SCALE: float = 1.0 / math.sqrt(8.0)
# float(kissing_points[0].pow(2).sum()) (castor.py:522): the origin-snap threshold.
C_SQ_NORM: float = 3.999999761581421


# ---------------------------------------------------------------------------
# Device plumbing
# ---------------------------------------------------------------------------
def _work_device(t: torch.Tensor) -> torch.device:
    if t.device.type == "cuda":
        return t.device
    if not torch.cuda.is_available():
        raise RuntimeError("pollux_b200 runs the H24 hot path on a CUDA device; none is available")
    return torch.device("cuda", torch.cuda.current_device())


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _call(dev: torch.device, name: str, *args) -> None:
    """Call libh24 with ``dev``'s context current (the library runs on the
    current device and the caller's current torch stream)."""
    with torch.cuda.device(dev):
        N.call(name, *args)


def _aligned(t: torch.Tensor) -> torch.Tensor:
    t = t.contiguous()
    return t if t.data_ptr() % 16 == 0 else t.clone()


# ---------------------------------------------------------------------------
# Codebook (castor.py:98-199, 263-266)
# ---------------------------------------------------------------------------
@lru_cache(maxsize=1)
def raw_kissing_points() -> torch.Tensor:
    """[196560, 24] int8 raw Leech coordinates in the reference's row order."""
    raw = np.empty((H24_KISSING_COUNT, H24_DIM), dtype=np.int8)
    N.call("h24_codebook_raw", raw.ctypes.data)
    return torch.from_numpy(raw)


@lru_cache(maxsize=1)
def _build_codebook_cpu() -> torch.Tensor:
    """[196561, 24] fp32 codebook; row 0 is the origin (castor.py:146-190).
    The fp32 values are raw * LEECH_SCALE rounded as torch rounds them."""
    kp = raw_kissing_points().to(torch.float32) * LEECH_SCALE
    return torch.cat([torch.zeros(1, H24_DIM, dtype=torch.float32), kp], dim=0)


def get_h24_codebook(device: torch.device | str, dtype: torch.dtype = torch.float16) -> torch.Tensor:
    """The 196,561-entry codebook on ``device`` (castor.py:193-199)."""
    return _build_codebook_cpu().to(device=device, dtype=dtype)


def codebook_fingerprint() -> tuple[float, ...]:
    """cb[:4,:4] as 16 floats, the .plx compatibility check (castor.py:263-266)."""
    return tuple(_build_codebook_cpu()[:4, :4].reshape(-1).tolist())


_VALIDATED: dict = {}


def _check_codebook(codebook: torch.Tensor) -> None:
    """The kernels search the fixed H24 table; refuse any other codebook."""
    if codebook.dim() != 2 or codebook.shape[0] != H24_CODEBOOK_COUNT or codebook.shape[1] != H24_DIM:
        raise ValueError(
            f"codebook must be the [{H24_CODEBOOK_COUNT}, {H24_DIM}] H24 table, got {tuple(codebook.shape)}")
    key = (codebook.data_ptr(), str(codebook.device), codebook.dtype, codebook._version)
    if key in _VALIDATED:
        return
    ref = _build_codebook_cpu().to(device=codebook.device, dtype=codebook.dtype)
    if not torch.equal(codebook, ref):
        raise ValueError("codebook differs from the H24 table that libh24 searches")
    if len(_VALIDATED) > 64:
        _VALIDATED.clear()
    _VALIDATED[key] = True


# ---------------------------------------------------------------------------
# Shape helpers (castor.py:269-306)
# ---------------------------------------------------------------------------
def h24_linear_atom_count(out_features: int, in_features: int) -> int:
    total = int(out_features) * int(in_features)
    if total % H24_DIM != 0:
        raise ValueError(
            f"H24 weight shape ({out_features}, {in_features}) has {total} params, "
            f"not divisible by H24_DIM={H24_DIM}.")
    return total // H24_DIM


def assert_h24_divisible(n_features: int, *, name: str = "features") -> None:
    if int(n_features) % H24_DIM != 0:
        raise ValueError(f"Pollux requires {name} divisible by H24_DIM={H24_DIM}; got {n_features}.")


def assert_row_aligned_width(d_model: int) -> None:
    assert_h24_divisible(d_model, name="d_model")


def assert_row_aligned_in_features(in_features: int) -> None:
    assert_h24_divisible(in_features, name="in_features")


def scale_bits_per_param(in_features: int) -> float:
    assert_row_aligned_in_features(in_features)
    return 16.0 / float(in_features)


def h24_linear_scale_row_count(out_features: int) -> int:
    return int(out_features)


# ---------------------------------------------------------------------------
# Row-RMS helpers (castor.py:309-339) -- elementwise torch ops, kept identical
# to the reference so that the training projection sees the same inputs.
# ---------------------------------------------------------------------------
def row_rms_from_matrix(weight: torch.Tensor) -> torch.Tensor:
    if weight.dim() != 2:
        raise ValueError(f"row_rms_from_matrix expects a 2D weight matrix, got {weight.dim()}D.")
    return torch.sqrt(weight.pow(2).mean(dim=-1) + NUMERICAL_EPSILON)


def normalize_matrix_by_row_rms(weight: torch.Tensor, sigma_rows: torch.Tensor | None = None):
    out_f, in_f = weight.shape
    assert_row_aligned_in_features(in_f)
    if sigma_rows is None:
        sigma_rows = row_rms_from_matrix(weight)
    sigma = sigma_rows.reshape(out_f, 1).clamp_min(NUMERICAL_EPSILON)
    return weight / sigma, sigma_rows.reshape(-1)


def scale_matrix_by_row_rms(weight: torch.Tensor, sigma_rows: torch.Tensor) -> torch.Tensor:
    out_f, _in_f = weight.shape
    return weight * sigma_rows.reshape(out_f, 1)


# ---------------------------------------------------------------------------
# 18-bit pack / unpack (castor.py:226-260)
# ---------------------------------------------------------------------------
def pack_indices(indices: torch.Tensor) -> torch.Tensor:
    """Pack 18-bit indices (4 per group) into 9 bytes big-endian."""
    flat = indices.reshape(-1)
    n = flat.numel()
    out_dev = flat.device
    groups = (n + 3) // 4
    if n == 0:
        return torch.zeros(0, dtype=torch.uint8, device=out_dev)
    dev = _work_device(flat)
    src = flat.to(dev)
    if src.dtype not in (torch.int32, torch.int64):
        src = src.to(torch.int32)  # the reference's .to(torch.int32)
    src = _aligned(src)
    out = torch.empty(groups * BYTES_PER_CHUNK, dtype=torch.uint8, device=dev)
    fn = "h24_pack_i64" if src.dtype == torch.int64 else "h24_pack"
    _call(dev, fn, src.data_ptr(), n, out.data_ptr(), _stream(dev))
    return out.to(out_dev)


def unpack_indices(packed: torch.Tensor, num_indices: int) -> torch.Tensor:
    """Unpack 9-byte big-endian groups back to 18-bit indices (int64)."""
    flat = packed.reshape(-1)
    if flat.dtype != torch.uint8:
        raise TypeError(f"packed indices must be uint8, got {flat.dtype}")
    if flat.numel() % BYTES_PER_CHUNK != 0:
        raise RuntimeError(
            f"shape '[-1, {BYTES_PER_CHUNK}]' is invalid for input of size {flat.numel()}")
    groups = flat.numel() // BYTES_PER_CHUNK
    n = len(range(4 * groups)[:num_indices])  # slice semantics of indices[:num_indices]
    out_dev = flat.device
    if n == 0:
        return torch.zeros(0, dtype=torch.int64, device=out_dev)
    dev = _work_device(flat)
    src = _aligned(flat.to(dev))
    out = torch.empty(n, dtype=torch.int64, device=dev)
    _call(dev, "h24_unpack_i64", src.data_ptr(), groups, n, out.data_ptr(), _stream(dev))
    return out.to(out_dev)


# ---------------------------------------------------------------------------
# Nearest codeword (castor.py:386-560)
# ---------------------------------------------------------------------------
def quantize_indices(x: torch.Tensor, rule: int = N.RULE_TRAIN) -> torch.Tensor:
    """int32 codebook indices of the atoms ``x`` ([..., 24], any float dtype),
    on the CUDA device that ran the search.  ``rule`` selects the origin test:
    RULE_TRAIN (2*max < c_sq_norm, castor.py:459) or RULE_PACK (||x|| < 1e-8,
    pack.py:174)."""
    xf = x.reshape(-1, H24_DIM)
    n = xf.shape[0]
    dev = _work_device(xf)
    out = torch.empty(n, dtype=torch.int32, device=dev)
    if n:
        # fp32 and bf16 atoms are read as they are (bf16 widens exactly, as
        # the reference's .float() does); other dtypes go through fp32.
        if xf.dtype == torch.bfloat16:
            xd, code = _aligned(xf.to(device=dev)), N.DTYPE_BF16
        else:
            xd, code = _aligned(xf.to(device=dev, dtype=torch.float32)), N.DTYPE_F32
        _call(dev, "h24_quantize_typed", xd.data_ptr(), n, code, int(rule), out.data_ptr(), _stream(dev))
    return out


def quantize_indices_many(xs: list[torch.Tensor], rule: int = N.RULE_TRAIN) -> list[torch.Tensor]:
    """quantize_indices for several tensors with one shared search pipeline
    (all on one CUDA device); returns one int32 index tensor per input."""
    if not xs:
        return []
    dev = _work_device(xs[0])
    flats = [_aligned(x.reshape(-1, H24_DIM).to(device=dev, dtype=torch.float32)) for x in xs]
    counts = [f.shape[0] for f in flats]
    out = torch.empty(sum(counts), dtype=torch.int32, device=dev)
    ptrs = (ctypes.c_void_p * len(flats))(*[f.data_ptr() for f in flats])
    cnts = (ctypes.c_int64 * len(flats))(*counts)
    _call(dev, "h24_quantize_segments", ctypes.cast(ptrs, ctypes.c_void_p),
          ctypes.cast(cnts, ctypes.c_void_p), len(flats), int(rule), out.data_ptr(), _stream(dev))
    return list(torch.split(out, counts))


_GATHER_DTYPES = {torch.float32: N.DTYPE_F32, torch.float16: N.DTYPE_F16, torch.bfloat16: N.DTYPE_BF16}


def _gather(idx: torch.Tensor, codebook: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    dev = idx.device
    code = _GATHER_DTYPES.get(dtype)
    if code is None:
        return codebook.to(device=dev, dtype=dtype).index_select(0, idx.long())
    out = torch.empty(idx.numel(), H24_DIM, dtype=dtype, device=dev)
    _call(dev, "h24_gather_codewords", idx.data_ptr(), idx.numel(), code, out.data_ptr(), _stream(dev))
    return out


def castor_quantize_leech(latent: torch.Tensor, codebook: torch.Tensor, chunk_size: int = 4096) -> torch.Tensor:
    """Nearest H24 codeword of every 24-D atom of ``latent`` (castor.py:487-560).

    Returns a tensor of the same shape and dtype as ``latent`` holding the
    codeword vectors.  The search is the exact fp64 argmax of x . kp with the
    lowest index on ties and the origin rule 2*max < c_sq_norm; ``chunk_size``
    is accepted for signature compatibility (the device kernels stream the
    codebook themselves).
    """
    orig_shape = latent.shape
    x = latent.reshape(-1, H24_DIM)
    if x.size(0) == 0:
        return latent.clone()
    _check_codebook(codebook)
    idx = quantize_indices(x, N.RULE_TRAIN)
    out = _gather(idx, codebook, latent.dtype)
    # One synchronisation per call, as the reference's own .item() has
    # (castor.py:522): a timed-out wait of the screen raises here instead of
    # returning unsearched codewords.
    device_check(idx.device)
    return out.view(orig_shape).to(latent.device)


def centers_to_indices(centers: torch.Tensor, codebook: torch.Tensor, chunk_size: int = 8192) -> torch.Tensor:
    """Nearest codebook index of each 24-D center (castor.py:202-223).

    All kissing points share one norm, so Euclidean nearest = training-rule
    argmax; it equals the reference's cdist argmin exactly for any vector that
    is a codebook entry (its documented use) and up to the 1e-7 relative norm
    spread of the fp32 table otherwise."""
    assert centers.dim() == 2 and centers.size(1) == H24_DIM
    assert codebook.dim() == 2 and codebook.size(1) == H24_DIM
    _check_codebook(codebook)
    return quantize_indices(centers, N.RULE_TRAIN).long().to(centers.device)


class CastorQuantizeLeech(torch.autograd.Function):
    """Straight-through wrapper of castor_quantize_leech (castor.py:563-580)."""

    @staticmethod
    def forward(ctx, latent: torch.Tensor, codebook: torch.Tensor) -> torch.Tensor:
        ctx.mark_non_differentiable(codebook)
        return castor_quantize_leech(latent, codebook)

    @staticmethod
    def backward(ctx, grad_output: torch.Tensor):
        return grad_output, None


# ---------------------------------------------------------------------------
# Instrumentation passthroughs
# ---------------------------------------------------------------------------
def device_check(device=None) -> None:
    """Raise if an earlier quantize call on ``device`` hit a bounded-wait timeout."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    _call(dev, "h24_check", _stream(dev))


def quantize_stats(device=None) -> tuple[int, int, int]:
    """(atoms resolved by the exhaustive scan, codewords scored exactly in
    fp64, 32-column units behind the screen's flags) since the last read."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    a, b, c = ctypes.c_int64(0), ctypes.c_int64(0), ctypes.c_int64(0)
    _call(dev, "h24_quantize_stats", ctypes.byref(a), ctypes.byref(b), ctypes.byref(c), _stream(dev))
    return int(a.value), int(b.value), int(c.value)


def launch_count() -> int:
    """Kernels libh24 has launched in this process."""
    return int(N.load().h24_launch_count())


def project_h24_many(pairs, sigma_out: bool = False, idx_out: bool = False):
    """The H24 projection block of pollux_step (pollux.py:874-884) for many
    parameters at once: for each (p_data, latent) pair of fp32 CUDA matrices,
    p_data <- (nearest codeword of latent / sigma / s_lattice) * sigma *
    s_lattice with sigma = row_rms_from_matrix(latent), in one fused pipeline
    (h24_project_layers).  Returns per pair a dict with the optional 'sigma'
    [rows] fp32 and 'idx' [rows*in/24] int32 tensors."""
    pairs = list(pairs)
    if not pairs:
        return []
    dev = _work_device(pairs[0][1])
    layers = (N.ProjectLayer * len(pairs))()
    keep, extras = [], []
    for i, (p, lat) in enumerate(pairs):
        if lat.dim() != 2 or p.shape != lat.shape:
            raise ValueError(f"p and latent must be matching 2-D matrices, got {tuple(p.shape)} and {tuple(lat.shape)}")
        rows, in_f = lat.shape
        assert_row_aligned_in_features(in_f)
        if p.dtype != torch.float32 or not p.is_contiguous() or p.device != dev:
            raise ValueError("p must be a contiguous fp32 tensor on the latent's device")
        l = _aligned(lat.detach().to(device=dev, dtype=torch.float32))
        ex = {}
        if sigma_out:
            ex["sigma"] = torch.empty(rows, dtype=torch.float32, device=dev)
        if idx_out:
            ex["idx"] = torch.empty(rows * in_f // H24_DIM, dtype=torch.int32, device=dev)
        keep.append(l)
        extras.append(ex)
        layers[i] = N.ProjectLayer(l.data_ptr(), p.data_ptr(), rows, in_f,
                                   ex["sigma"].data_ptr() if sigma_out else None,
                                   ex["idx"].data_ptr() if idx_out else None)
    _call(dev, "h24_project_layers", ctypes.cast(layers, ctypes.c_void_p), len(pairs), _stream(dev))
    return extras


def project_h24_(p_data: torch.Tensor, latent: torch.Tensor) -> torch.Tensor:
    """In-place p_data.copy_(center) of pollux_step's H24 block for one
    parameter (see project_h24_many); returns p_data."""
    project_h24_many([(p_data, latent)])
    return p_data
