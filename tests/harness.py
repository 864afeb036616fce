"""Helpers shared by the GPU parity tests: seeded inputs, device copies in the
activation dtype, and side-by-side sessions on the CUDA path (through the C
ABI) and the oracle."""
from __future__ import annotations

import numpy as np

import ndattn
import ndoracle as O

TOL = 1e-3   # max |gpu - oracle| <= TOL * max(1, |oracle|): the north-star bound vs fp32/fp64 reference


def torch_dtype(dt):
    import torch
    return {O.F32: torch.float32, O.F16: torch.float16, O.BF16: torch.bfloat16}[dt]


def dev(x: np.ndarray, act_dt: int):
    """Device tensor of dtype act_dt holding exactly round_act(x, act_dt)."""
    import torch
    return torch.from_numpy(np.ascontiguousarray(O.round_act(x, act_dt))).to("cuda").to(torch_dtype(act_dt))


def rel_err(got, want) -> float:
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    assert got.shape == want.shape, (got.shape, want.shape)
    return float(np.max(np.abs(got - want) / np.maximum(1.0, np.abs(want)))) if want.size else 0.0


def kv_np_dtype(kv_dt):
    return {O.I8: np.int8, O.F32: np.float32, O.F16: np.float16, O.BF16: np.uint16}[kv_dt]


def random_kv_rows(rng, n, width, kv_dt, scale=0.5, peaky_rows=None):
    """Synthetic cache rows stored as kv_dt (plus int8 scales)."""
    x = (rng.standard_normal((n, width)) * scale).astype(np.float32)
    if peaky_rows is not None:
        x[peaky_rows] *= 8.0
    if kv_dt == O.F32:
        return x, None
    if kv_dt == O.F16:
        return x.astype(np.float16), None
    if kv_dt == O.BF16:
        return O.to_bf16_bits(x), None
    raise ValueError("int8 rows come from the quantiser, not from here")


def cache_bits(a: np.ndarray) -> np.ndarray:
    """Raw element bits for exact comparisons (f16 -> u16, f32 -> u32)."""
    if a.dtype == np.float16:
        return a.view(np.uint16)
    if a.dtype == np.float32:
        return a.view(np.uint32)
    return a


def oracle_cache(seq: O._SeqBase, layer: int, kv_dt):
    """Oracle cache of one layer as the library's read_cache returns it."""
    k, v = seq.k[layer], seq.v[layer]
    if kv_dt == O.F16:
        k, v = k.view(np.float16), v.view(np.float16)
    return k, v
