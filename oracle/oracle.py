"""CPU oracle for the H24 hot path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may import this module, and only as the checker or as the timed CPU
baseline.  The product (``pollux_b200``) never calls it and has no CPU fallback.

It wraps ``oracle/h24_oracle.c`` (built by ``oracle/Makefile`` into
``oracle/_build/libh24_oracle.so``) and adds numpy restatements of the
reference's three nearest-codeword semantics:

* ``nearest_exact``   -- fp64 argmax of x.kp, lowest index on ties
                         (the parity judge; C, multithreaded).
* ``nearest_fp32_pack_rule`` -- fp32 ``atoms @ kp.T``, first max, zero only for
                         ``||atom|| < 1e-8`` (restates pack.py:139-180).
* ``nearest_bf16_train_rule`` -- scores of bf16-rounded atoms against the
                         codebook in fp32, origin snap ``2*max < c_sq_norm``
                         (restates the Triton kernel castor.py:386-462 and the
                         autocast fallback castor.py:549-557 up to score
                         rounding).

Pack / unpack / dequant restate castor.py:226-260 and pollux.py:485-500.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading
from functools import lru_cache

import numpy as np

H24_DIM = 24
H24_KISSING_COUNT = 196_560
H24_CODEBOOK_COUNT = 196_561
C_SQ_NORM = 3.999999761581421          # castor.py:522 (measured on the reference)
RULE_TRAIN = 0                          # origin iff 2*max < C_SQ_NORM
RULE_PACK = 1                           # origin iff ||x|| < 1e-8

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libh24_oracle.so")
_lock = threading.Lock()


def build() -> str:
    """Compile the C oracle (idempotent) and return the library path."""
    with _lock:
        src = os.path.join(_HERE, "h24_oracle.c")
        if (not os.path.exists(_LIB_PATH)
                or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src)):
            subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


@lru_cache(maxsize=1)
def lib() -> ctypes.CDLL:
    path = build()
    L = ctypes.CDLL(path)
    P = ctypes.c_void_p
    i64 = ctypes.c_int64
    L.h24o_raw_kissing_points.argtypes = [P]
    L.h24o_raw_kissing_points.restype = ctypes.c_int
    L.h24o_codebook_f32.argtypes = [P]
    L.h24o_codebook_f32.restype = ctypes.c_int
    L.h24o_nearest.argtypes = [P, P, i64, ctypes.c_int, P, P, ctypes.c_int]
    L.h24o_nearest.restype = None
    L.h24o_pack.argtypes = [P, i64, P]
    L.h24o_pack.restype = None
    L.h24o_unpack.argtypes = [P, i64, i64, P]
    L.h24o_unpack.restype = None
    L.h24o_dequant.argtypes = [P, P, P, i64, i64, P]
    L.h24o_dequant.restype = i64
    L.h24o_score.argtypes = [P, P, ctypes.c_int32]
    L.h24o_score.restype = ctypes.c_double
    L.h24o_sigma16_from_rms.argtypes = [ctypes.c_float]
    L.h24o_sigma16_from_rms.restype = ctypes.c_uint16
    return L


def _ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


# ---------------------------------------------------------------------------
# Codebook (castor.py:98-199)
# ---------------------------------------------------------------------------
@lru_cache(maxsize=1)
def raw_kissing_points() -> np.ndarray:
    """[196560, 24] int8 raw coordinates, in the reference's sorted order."""
    out = np.empty((H24_KISSING_COUNT, H24_DIM), dtype=np.int8)
    rc = lib().h24o_raw_kissing_points(_ptr(out))
    if rc != 0:
        raise RuntimeError(f"oracle codebook generation failed (rc={rc})")
    out.setflags(write=False)
    return out


@lru_cache(maxsize=1)
def codebook_f32() -> np.ndarray:
    """[196561, 24] fp32 codebook, origin at row 0 (get_h24_codebook fp32)."""
    out = np.empty((H24_CODEBOOK_COUNT, H24_DIM), dtype=np.float32)
    rc = lib().h24o_codebook_f32(_ptr(out))
    if rc != 0:
        raise RuntimeError(f"oracle codebook generation failed (rc={rc})")
    out.setflags(write=False)
    return out


def kissing_points_f32() -> np.ndarray:
    return codebook_f32()[1:]


def fingerprint() -> tuple:
    """codebook_fingerprint(): cb[:4,:4] as 16 floats (castor.py:263-266)."""
    return tuple(float(v) for v in codebook_f32()[:4, :4].reshape(-1))


# ---------------------------------------------------------------------------
# Nearest codeword
# ---------------------------------------------------------------------------
def nearest_exact(x: np.ndarray, rule: int = RULE_TRAIN, nthreads: int = 0,
                  return_best: bool = False):
    """Exact fp64 nearest codeword index for each row of x ([n,24] fp32)."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, H24_DIM)
    n = x.shape[0]
    idx = np.empty(n, dtype=np.int32)
    best = np.empty(n, dtype=np.float64)
    kp = np.ascontiguousarray(kissing_points_f32())
    if n:
        lib().h24o_nearest(_ptr(kp), _ptr(x), n, int(rule), _ptr(idx), _ptr(best), int(nthreads))
    return (idx, best) if return_best else idx


def scores_fp64(x: np.ndarray, idx: np.ndarray) -> np.ndarray:
    """fp64 score x.kp[idx-1] (0 for the origin), same fma order as the GPU."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, H24_DIM)
    cb = codebook_f32().astype(np.float64)
    c = cb[np.asarray(idx, dtype=np.int64)]
    acc = np.zeros(x.shape[0], dtype=np.float64)
    xd = x.astype(np.float64)
    for i in range(H24_DIM):
        acc = acc + xd[:, i] * c[:, i]   # products exact in fp64
    return acc


def dist2_fp64(x: np.ndarray, idx: np.ndarray) -> np.ndarray:
    """Squared distance ||x - cb[idx]||^2 in fp64."""
    x = np.asarray(x, dtype=np.float32).reshape(-1, H24_DIM).astype(np.float64)
    c = codebook_f32().astype(np.float64)[np.asarray(idx, dtype=np.int64)]
    return ((x - c) ** 2).sum(axis=1)


def nearest_fp32_pack_rule(atoms: np.ndarray, chunk: int = 4096) -> np.ndarray:
    """Restates pack._quantize_h24_layer's search (pack.py:166-177) in numpy:
    fp32 scores, first maximum, index 0 only when ||atom||_2 < 1e-8."""
    a = np.ascontiguousarray(atoms, dtype=np.float32).reshape(-1, H24_DIM)
    kpT = np.ascontiguousarray(kissing_points_f32().T)
    out = np.zeros(a.shape[0], dtype=np.int64)
    for i in range(0, a.shape[0], chunk):
        s = a[i:i + chunk]
        scores = s @ kpT
        best = scores.argmax(axis=1) + 1
        zero = np.linalg.norm(s, axis=1) < np.float32(1e-8)
        best[zero] = 0
        out[i:i + chunk] = best
    return out


def to_bf16(x: np.ndarray) -> np.ndarray:
    """Round fp32 to bf16 (round to nearest even), returned as fp32."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return r.astype(np.uint32).view(np.float32).reshape(np.shape(x))


def nearest_bf16_train_rule(x: np.ndarray, chunk: int = 4096) -> np.ndarray:
    """bf16(x) . bf16(kp) accumulated in fp32, lowest index among maxima,
    origin iff 2*max < c_sq_norm (castor.py:436-462)."""
    a = to_bf16(np.asarray(x, dtype=np.float32).reshape(-1, H24_DIM))
    kpT = np.ascontiguousarray(to_bf16(kissing_points_f32()).T)
    out = np.zeros(a.shape[0], dtype=np.int64)
    for i in range(0, a.shape[0], chunk):
        scores = a[i:i + chunk] @ kpT
        best = scores.argmax(axis=1)
        m = scores[np.arange(scores.shape[0]), best]
        r = best + 1
        r[(2.0 * m) < np.float32(C_SQ_NORM)] = 0
        out[i:i + chunk] = r
    return out


# ---------------------------------------------------------------------------
# Pack / unpack (castor.py:226-260)
# ---------------------------------------------------------------------------
def pack_indices(indices: np.ndarray) -> np.ndarray:
    """numpy restatement of castor.pack_indices: 4 x 18 bit -> 9 bytes."""
    v = np.asarray(indices).reshape(-1).astype(np.int64).astype(np.int32)  # .to(int32) wraps
    rem = v.size % 4
    if rem:
        v = np.concatenate([v, np.zeros(4 - rem, dtype=np.int32)])
    g = v.reshape(-1, 4)
    i0, i1, i2, i3 = g[:, 0], g[:, 1], g[:, 2], g[:, 3]
    out = np.empty((g.shape[0], 9), dtype=np.uint8)
    out[:, 0] = (i0 >> 10) & 0xFF
    out[:, 1] = (i0 >> 2) & 0xFF
    out[:, 2] = ((i0 & 0x03) << 6) | ((i1 >> 12) & 0x3F)
    out[:, 3] = (i1 >> 4) & 0xFF
    out[:, 4] = ((i1 & 0x0F) << 4) | ((i2 >> 14) & 0x0F)
    out[:, 5] = (i2 >> 6) & 0xFF
    out[:, 6] = ((i2 & 0x3F) << 2) | ((i3 >> 16) & 0x03)
    out[:, 7] = (i3 >> 8) & 0xFF
    out[:, 8] = i3 & 0xFF
    return out.reshape(-1)


def unpack_indices(packed: np.ndarray, num_indices: int) -> np.ndarray:
    """numpy restatement of castor.unpack_indices (int64 result)."""
    c = np.asarray(packed, dtype=np.uint8).reshape(-1, 9).astype(np.int32)
    i0 = (c[:, 0] << 10) | (c[:, 1] << 2) | (c[:, 2] >> 6)
    i1 = ((c[:, 2] & 0x3F) << 12) | (c[:, 3] << 4) | (c[:, 4] >> 4)
    i2 = ((c[:, 4] & 0x0F) << 14) | (c[:, 5] << 6) | (c[:, 6] >> 2)
    i3 = ((c[:, 6] & 0x03) << 16) | (c[:, 7] << 8) | c[:, 8]
    return np.stack([i0, i1, i2, i3], axis=1).reshape(-1)[:num_indices].astype(np.int64)


def pack_indices_c(indices: np.ndarray) -> np.ndarray:
    v = np.ascontiguousarray(np.asarray(indices).reshape(-1).astype(np.int64).astype(np.int32))
    out = np.empty(((v.size + 3) // 4) * 9, dtype=np.uint8)
    if v.size:
        lib().h24o_pack(_ptr(v), v.size, _ptr(out))
    return out


def unpack_indices_c(packed: np.ndarray, num_indices: int) -> np.ndarray:
    p = np.ascontiguousarray(packed, dtype=np.uint8).reshape(-1)
    groups = p.size // 9
    n = min(int(num_indices), 4 * groups)
    out = np.empty(max(n, 0), dtype=np.int32)
    if n > 0:
        lib().h24o_unpack(_ptr(p), groups, n, _ptr(out))
    return out.astype(np.int64)


# ---------------------------------------------------------------------------
# Dequant (pollux.py:485-500) and the pack-rule row scale (pack.py:164)
# ---------------------------------------------------------------------------
def dequant(packed: np.ndarray, sigma16: np.ndarray, rows: int, in_features: int) -> np.ndarray:
    """fp16 [rows, in_features] weight rebuilt like PackedH24Linear.materialize."""
    p = np.ascontiguousarray(packed, dtype=np.uint8).reshape(-1)
    s = np.ascontiguousarray(sigma16, dtype=np.float16).reshape(-1)
    out = np.empty((rows, in_features), dtype=np.float16)
    cb = np.ascontiguousarray(codebook_f32())
    bad = lib().h24o_dequant(_ptr(cb), _ptr(p), _ptr(s.view(np.uint16)), rows, in_features,
                             _ptr(out.view(np.uint16)))
    if bad:
        raise ValueError(f"{bad} packed indices exceed the codebook")
    return out


def dequant_numpy(packed: np.ndarray, sigma16: np.ndarray, rows: int, in_features: int) -> np.ndarray:
    """Same as ``dequant`` with numpy's fp16 arithmetic (two roundings)."""
    atoms = rows * in_features // H24_DIM
    idx = unpack_indices(packed, atoms)
    cb16 = codebook_f32().astype(np.float16)[idx].reshape(rows, in_features // H24_DIM, H24_DIM)
    s16 = np.asarray(sigma16, dtype=np.float16).reshape(-1, 1, 1)
    t = (cb16.astype(np.float32) * s16.astype(np.float32)).astype(np.float16)
    w = (t.astype(np.float32) * np.float32(0.7071067811865476)).astype(np.float16)
    return w.reshape(rows, in_features)


# Row scales.  The reference computes sigma = sqrt(w.pow(2).mean(-1) + 1e-8)
# (castor.py:309-313) and sigma16 = fp16(clamp_min(sigma * sqrt(12), 1e-8))
# (pack.py:164) with torch ops, so the fp32 mean depends on the device torch
# reduces on.  Restated here for both devices of the reference:
#   * CUDA (pack.py's default --device): torch's CUDA reduction order, from
#     PyTorch 2.11's ATen/native/cuda/Reduce.cuh (setReduceConfig,
#     input_vectorized_thread_reduce_impl, thread_reduce_impl, block_x_reduce,
#     block_y_reduce) and MeanOps (ATen/native/SharedReduceOps.h): mean =
#     sum * (fp32(rows) / fp32(rows * n)); restated in numpy below;
#   * CPU: the same torch expression run on CPU tensors (torch's CPU mean is a
#     cascade sum divided by n).
def _last_pow2(v: int) -> int:
    p = 1
    while p * 2 <= v:
        p *= 2
    return p


def torch_cuda_mean_plan(rows: int, n: int) -> dict:
    """Launch plan torch's CUDA reduction picks for mean(dim=-1) of a
    contiguous fp32 [rows, n] tensor (Reduce.cuh setReduceConfig, vt0 = 4)."""
    vec = n >= 128
    dim0 = n // 4 if vec else n
    d0 = _last_pow2(dim0) if dim0 < 512 else 512
    d1 = _last_pow2(rows) if rows < 512 else 512
    bw = min(d0, 32)
    bh = min(d1, 512 // bw)
    bw = min(d0, 512 // bh)
    vpt = -(-n // bw)
    split = vpt >= min(16 * bh, 256)
    factor = np.float32(np.float32(rows) / np.float32(rows * n))
    return {"vec": vec, "bw": bw, "bh": bh, "split": split, "factor": factor}


def _tree(v: np.ndarray, width: int) -> np.ndarray:
    """Column 0 of the halving tree v[:, :off] += v[:, off:2 off] over the
    first `width` columns (width a power of two), in fp32."""
    v = v[:, :width].copy()
    off = width // 2
    while off > 0:
        v[:, :off] = v[:, :off] + v[:, off:2 * off]
        off //= 2
    return v[:, 0]


def row_sumsq_cuda_order(w: np.ndarray, matrix_rows: int | None = None, first_row: int = 0) -> np.ndarray:
    """fp32 sum of squares of each row in torch's CUDA mean order; the rows are
    rows first_row.. of a matrix of matrix_rows rows (default: just these)."""
    sq = np.asarray(w, dtype=np.float32)
    sq = (sq * sq).astype(np.float32)
    R, n = sq.shape
    plan = torch_cuda_mean_plan(matrix_rows if matrix_rows is not None else R, n)
    bw, bh, split = plan["bw"], plan["bh"], plan["split"]
    lanes = bw * bh if split else bw       # thread t = x + y * bw shares the row
    out = np.empty(R, dtype=np.float32)
    if plan["vec"]:
        shifts = ((first_row + np.arange(R)) * n) % 4
        for shift in np.unique(shifts):
            rows_s = np.nonzero(shifts == shift)[0]
            x = sq[rows_s]
            acc = np.zeros((len(rows_s), lanes, 4), dtype=np.float32)
            base = 0
            if shift:
                base = 4 - int(shift)
                for t in range(int(shift), 4):          # head: lanes shift..3 of y = 0
                    acc[:, t, 0] = x[:, t - int(shift)]
            end = n - base
            nvec = end // 4
            xv = x[:, base:base + 4 * nvec].reshape(len(rows_s), nvec, 4)
            for i0 in range(0, nvec, lanes):
                i1 = min(i0 + lanes, nvec)
                acc[:, :i1 - i0, :] = acc[:, :i1 - i0, :] + xv[:, i0:i1, :]
            tail = end - end % 4
            for t in range(end % 4):                   # tail: lanes 0.. of y = 0
                acc[:, t, 0] = acc[:, t, 0] + x[:, base + tail + t]
            v = ((acc[:, :, 0] + acc[:, :, 1]) + acc[:, :, 2]) + acc[:, :, 3]
            out[rows_s] = _combine_lanes(v, bw, bh, split)
    else:
        acc = np.zeros((R, lanes, 4), dtype=np.float32)
        for t in range(lanes):
            i = t
            while i + 3 * lanes < n:
                for k in range(4):
                    acc[:, t, k] = acc[:, t, k] + sq[:, i + k * lanes]
                i += 4 * lanes
            for k in range(4):
                if i >= n:
                    break
                acc[:, t, k] = acc[:, t, k] + sq[:, i]
                i += lanes
        v = ((acc[:, :, 0] + acc[:, :, 1]) + acc[:, :, 2]) + acc[:, :, 3]
        out = _combine_lanes(v, bw, bh, split)
    return out


def _combine_lanes(v: np.ndarray, bw: int, bh: int, split: bool) -> np.ndarray:
    """block_x_reduce (shared memory down to 32 lanes, then shuffles with
    halving offsets) per block row, then block_y_reduce when the block rows
    share a matrix row."""
    groups = bh if split else 1
    heads = []
    for y in range(groups):
        g = v[:, y * bw:(y + 1) * bw]
        if bw > 32:
            g = g.copy()
            off = bw // 2
            while off >= 32:
                g[:, :off] = g[:, :off] + g[:, off:2 * off]
                off //= 2
            heads.append(_tree(g, 32))
        else:
            heads.append(_tree(g, bw))
    if not split:
        return heads[0]
    return _tree(np.stack(heads, axis=1), bh)


def row_rms_cuda_order(weight: np.ndarray, matrix_rows: int | None = None, first_row: int = 0) -> np.ndarray:
    """castor.row_rms_from_matrix (castor.py:309-313) as torch computes it on
    a CUDA tensor: fp32 sqrt(sum * factor + 1e-8)."""
    w = np.asarray(weight, dtype=np.float32)
    plan = torch_cuda_mean_plan(matrix_rows if matrix_rows is not None else w.shape[0], w.shape[1])
    mean = (row_sumsq_cuda_order(w, matrix_rows, first_row) * plan["factor"]).astype(np.float32)
    return np.sqrt((mean + np.float32(1e-8)).astype(np.float32)).astype(np.float32)


def sigma16_from_rms(rms: np.ndarray) -> np.ndarray:
    """pack.py:164 after the row RMS: fp16(clamp_min(rms * fp32(sqrt 12), 1e-8)),
    NaN kept."""
    s = (np.asarray(rms, dtype=np.float32) * np.float32(np.sqrt(12.0))).astype(np.float32)
    s = np.where(np.isnan(s), s, np.maximum(s, np.float32(1e-8)))
    return s.astype(np.float16)


def sigma16_pack_rule(weight: np.ndarray, matrix_rows: int | None = None, first_row: int = 0) -> np.ndarray:
    """fp16 row scales of pack.py:164 as the reference computes them on its
    default CUDA device (torch's CUDA mean order)."""
    return sigma16_from_rms(row_rms_cuda_order(weight, matrix_rows, first_row))


def sigma16_pack_rule_cpu_torch(weight) -> np.ndarray:
    """fp16 row scales of pack.py:164 with the reference's torch expression run
    on CPU tensors (the reference with --device cpu)."""
    import torch
    w = torch.as_tensor(np.asarray(weight)).float()
    rms = torch.sqrt(w.pow(2).mean(dim=-1) + 1e-8)
    return (rms * float(np.sqrt(12.0))).clamp_min(1e-8).to(torch.float16).numpy()


def int8_quantize(weight: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """numpy restatement of pack._quantize_int8 (pack.py:124-136): per row
    mu = max(max|w|, fp32(1e-8)) in fp32, q = clamp(round_half_even(
    fp32(fp32(w / mu) * 127)), -128, 127) as int8 (NaN -> 0), mu as fp16."""
    w = np.asarray(weight, dtype=np.float32)
    with np.errstate(invalid="ignore", divide="ignore", over="ignore"):
        mu = np.max(np.abs(w), axis=-1, keepdims=True)        # NaN propagates
        mu = np.where(np.isnan(mu), mu, np.maximum(mu, np.float32(1e-8)))
        t = (w / mu).astype(np.float32) * np.float32(127.0)
        r = np.clip(np.rint(t), -128, 127)
        q = np.where(np.isnan(r), 0, r).astype(np.int8)
        return q, mu[..., 0].astype(np.float16)


def int8_dequant(q: np.ndarray, mu16: np.ndarray) -> np.ndarray:
    """numpy restatement of PackedInt8Embedding/Linear.materialize
    (pollux.py:519-523): fp16(q * fp16(fp32(mu) / 127)), both roundings."""
    with np.errstate(invalid="ignore", over="ignore"):
        s = (np.asarray(mu16, dtype=np.float16).astype(np.float32) / np.float32(127.0)).astype(np.float16)
        return (np.asarray(q).astype(np.float32) * s.astype(np.float32)[..., None]).astype(np.float16)
