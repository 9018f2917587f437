"""int8 group quantisation restated in numpy (test infrastructure only).

Restates the reference's "q8" weight format (engine/kernels.js:1-47):
  * weights are symmetric int8 with one f32 scale per group of G consecutive values along a row
    (kernels.js:5 fixes G = 128; G = K, one scale per output row, is the per-row absmax variant);
  * scale = absmax / 127, or 1 when the group is all zeros (kernels.js:39-40);
  * q = round(v / scale), round half to even (WGSL `round`), stored as two's complement bytes
    (kernels.js:41-42, packed four per u32, little endian, which is the same bytes as a row-major int8 array);
  * dequantised value = f32(q) * scale (kernels.js:7-11 sign-extending unpack, kernels.js:74-75 `q4(w) * s`).

The division is IEEE-754 f32 division, correctly rounded.  That is the contract the CUDA quantiser meets bit for bit
(WGSL itself only promises 2.5 ulp for `/`).
"""
import numpy as np


def quantize(w, group):
    """W[N, K] (any float dtype, converted to f32 first, as kernels.js:26-30 does) -> (q int8[N, K], s f32[N, K/G]).

    kernels.js:16-47: one group of `group` values per workgroup; absmax by tree reduction (exact: max is
    order-independent), scale = m / 127 (1 if m == 0), q = round(v / scale).
    """
    w = np.ascontiguousarray(np.asarray(w, dtype=np.float32))
    n, k = w.shape
    if group <= 0 or k % group:
        raise ValueError(f"K={k} is not a multiple of the group size {group}")
    g = w.reshape(n, k // group, group)
    m = np.abs(g).max(axis=2)
    scale = np.where(m == 0, np.float32(1.0), m / np.float32(127.0)).astype(np.float32)
    r = np.rint(g / scale[:, :, None]).astype(np.int32)  # np.rint: round half to even, like WGSL round()
    q = r.astype(np.int8).reshape(n, k)  # two's complement low byte (kernels.js:42 `u32(r) & 0xff`)
    return q, scale


def dequantize(q, s, group):
    """(q int8[N, K], s f32[N, K/G]) -> f32[N, K] with f32(q) * scale per element (kernels.js:74-75)."""
    n, k = q.shape
    return (q.astype(np.float32).reshape(n, k // group, group) * s[:, :, None].astype(np.float32)).reshape(n, k)


def matvec(x, q, s, group, y=None):
    """y[M, N] (+)= x[M, K] . dequant(W)[N, K]^T (kernels.js:55-94 matvec, kernels.js:97-151 matmul).

    Accumulates in float64 so the result is the exact dot product of the f32 operands rounded once; the GPU kernels
    are compared against it with a tolerance that covers f32 summation order.
    """
    wd = dequantize(q, s, group).astype(np.float64)
    out = np.asarray(x, dtype=np.float64) @ wd.T
    if y is not None:
        out = out + np.asarray(y, dtype=np.float64)
    return out.astype(np.float32)


def gather(ids, q, s, group, mul=1.0):
    """Embedding lookup y[t, :] = dequant(E)[ids[t], :] * mul (kernels.js:205-221).

    kernels.js:219 computes q * (scale * mul); with mul == 1 this is exactly f32(q) * scale.
    """
    ids = np.asarray(ids, dtype=np.int64)
    rows = q[ids].astype(np.float32)
    sc = (s[ids].astype(np.float32) * np.float32(mul)).astype(np.float32)
    n, k = rows.shape
    return (rows.reshape(n, k // group, group) * sc[:, :, None]).reshape(n, k)
