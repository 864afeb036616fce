"""ndattn - Python view of the C ABI in include/nd_attn.h (libndattn.so).

The engine-facing surface is the C ABI; this module is the thin host mirror
the tests and the benchmark use. It mirrors the reference engine's session
calls (engine/include/nd_model.h:191-236: reset, set_sink, snapshot, rewind,
prefix_save/restore/free) and its attention seam (the static attention() of
engine/src/nd_model.c:2382, lines 2419-2483), with the same argument meaning
and the same error behaviour: negative return codes become NdAttnError, a
prefix that belongs to another handle is refused (code -1), a failed
prefix_save returns None like the reference's NULL.

Tensor arguments of the device entry points are torch CUDA tensors (or raw
device addresses as int); the *_host entry points take numpy arrays. There is
no CPU fallback: importing works anywhere, but opening a handle needs the
compiled library and an sm_100 GPU, and fails loudly otherwise.
"""
from __future__ import annotations

import ctypes
import os
import re
from ctypes import POINTER, c_char_p, c_float, c_int, c_int32, c_size_t, c_uint32, c_uint64, c_void_p

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libndattn.so")
HEADER_PATH = os.path.join(os.path.dirname(HERE), "include", "nd_attn.h")
HEADER_PATHS = [HEADER_PATH, os.path.join(os.path.dirname(HERE), "include", "nd_cq.h")]

DT_I8, DT_F32, DT_F16, DT_BF16 = 0, 1, 2, 3
DT_NAMES = {"i8": DT_I8, "int8": DT_I8, "f32": DT_F32, "float32": DT_F32, "f16": DT_F16,
            "float16": DT_F16, "bf16": DT_BF16, "bfloat16": DT_BF16}
ERR_ARG, ERR_GEOM, ERR_NOMEM, ERR_CUDA, ERR_RANGE, ERR_TIMEOUT, ERR_NOGPU = -1, -10, -12, -14, -15, -16, -17
NOALLOC_MAX_ITEMS = 16384            # ND_ATTN_NOALLOC_MAX_ITEMS
GATHER_BLOB_BYTES = 128              # ND_ATTN_GATHER_BLOB_BYTES


class NdAttnError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"nd_attn error {code}: {msg}")
        self.code = code


class Config(ctypes.Structure):
    _fields_ = [("n_layers", c_uint32), ("n_heads", c_uint32), ("n_kv_heads", c_uint32),
                ("qk_head_dim", c_uint32), ("v_head_dim", c_uint32), ("window", c_uint32),
                ("max_seqs", c_uint32), ("block_size", c_uint32), ("n_blocks", c_uint32),
                ("max_pos", c_uint32), ("rope_theta", c_float), ("kv_dtype", c_int32),
                ("act_dtype", c_int32), ("out_dtype", c_int32), ("device", c_int32),
                ("qkv_conv_taps", c_uint32)]


class CqTensor(ctypes.Structure):
    """nd_cq_tensor (include/nd_cq.h): one decoded .cact directory record."""
    _fields_ = [("dtype", ctypes.c_uint8), ("ndim", ctypes.c_uint8), ("shape", c_uint32 * 4),
                ("offset", c_uint64), ("nbytes", c_uint64), ("group", c_uint32), ("bits", c_uint32)]


# Per-layer slots of a .cact archive (bind_layer, engine/src/nd_model.c:646-654).
CQ_SLOTS = ["norm_in", "q_proj", "k_proj", "v_proj", "q_taps", "k_taps", "v_taps", "q_norm", "k_norm",
            "gate_proj", "out_proj", "post_norm", "attn_gate", "pre_hada", "d1", "d2", "b2", "d3", "d4",
            "w1a", "w1b", "w2a", "w2b", "w3a", "w3b", "cond_v", "cond_u"]

_lib = None


def header_functions(paths=None) -> list[str]:
    """Names of every entry point include/nd_attn.h and include/nd_cq.h declare."""
    names = set()
    for path in paths or HEADER_PATHS:
        src = open(path).read()
        names |= set(re.findall(r"^ND_ATTN_API\s+[^(;]*?\b(nd_(?:attn|cq)_\w+)\s*\(", src, re.M))
    return sorted(names)


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    """Loads libndattn.so (built by `make -C esp32-needle-3_b200`)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise FileNotFoundError(f"{path} is missing: build it with `make -C {HERE}` (no CPU fallback exists)")
    lib = ctypes.CDLL(path)
    vp, u32, u32p = c_void_p, c_uint32, POINTER(c_uint32)
    sig = {
        "nd_attn_config_init": (None, [POINTER(Config)]),
        "nd_attn_open": (c_int, [POINTER(Config), POINTER(vp)]),
        "nd_attn_close": (None, [vp]),
        "nd_attn_set_head_norm": (c_int, [vp, u32, vp, vp]),
        "nd_attn_set_conv_taps": (c_int, [vp, u32, vp, vp, vp]),
        "nd_attn_reset": (c_int, [vp, u32]),
        "nd_attn_set_sink": (c_int, [vp, u32, u32]),
        "nd_attn_snapshot": (c_int, [vp, u32]),
        "nd_attn_rewind": (c_int, [vp, u32]),
        "nd_attn_advance": (c_int, [vp, u32, vp, vp]),
        "nd_attn_get_state": (c_int, [vp, u32, u32p, u32p]),
        "nd_attn_set_state": (c_int, [vp, u32, u32, u32]),
        "nd_attn_decode": (c_int, [vp, u32, u32, vp, vp, vp, vp, vp, vp]),
        "nd_attn_prefill": (c_int, [vp, u32, u32, vp, vp, vp, vp, vp, vp, vp]),
        "nd_attn_rope_append": (c_int, [vp, u32, u32, vp, vp, vp, vp, vp]),
        "nd_attn_decode_host": (c_int, [vp, u32, u32, vp, vp, vp, vp, vp, vp]),
        "nd_attn_decode_noalloc": (c_int, [vp, u32, u32, vp, vp, vp, vp, vp]),
        "nd_attn_decode_shared": (c_int, [vp, u32, u32, vp, u32, u32, vp, vp, vp, vp, vp]),
        "nd_attn_gather_check": (c_int, [vp, u32, u32]),
        "nd_attn_gather_init": (c_int, [vp, u32, u32, vp]),
        "nd_attn_gather_attach": (c_int, [vp, vp]),
        "nd_attn_decode_gather": (c_int, [vp, u32, u32, vp, vp, vp, vp, vp, vp]),
        "nd_attn_prefill_host": (c_int, [vp, u32, u32, vp, vp, vp, vp, vp, vp, vp]),
        "nd_attn_prefix_save": (vp, [vp, u32]),
        "nd_attn_prefix_restore": (c_int, [vp, u32, vp]),
        "nd_attn_prefix_free": (None, [vp]),
        "nd_attn_prefix_read": (c_int, [vp, vp, c_size_t, POINTER(c_size_t), u32p, u32p]),
        "nd_attn_read_cache": (c_int, [vp, u32, u32, u32, u32, vp, vp, vp, vp]),
        "nd_attn_write_cache": (c_int, [vp, u32, u32, u32, u32, vp, vp, vp, vp]),
        "nd_attn_set_block_table": (c_int, [vp, u32, vp]),
        "nd_attn_sync": (c_int, [vp]),
        "nd_attn_selftest_wait": (c_int, [vp, u32]),
        "nd_attn_stream": (vp, [vp]),
        "nd_cq_open": (c_int, [vp, c_size_t, c_int, POINTER(vp)]),
        "nd_cq_close": (None, [vp]),
        "nd_cq_header": (c_int, [vp, vp]),
        "nd_cq_tensor_info": (c_int, [vp, u32, POINTER(CqTensor)]),
        "nd_cq_layer_tensor": (c_int, [vp, u32, u32, u32p]),
        "nd_cq_read_f32": (c_int, [vp, u32, vp, c_size_t]),
        "nd_cq_project": (c_int, [vp, u32, vp, u32, vp, vp, vp]),
        "nd_attn_set_stream": (c_int, [vp, vp]),
        "nd_attn_launch_count": (c_uint64, [vp]),
        "nd_attn_last_error": (c_char_p, []),
        "nd_attn_version": (c_char_p, []),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def gather_check(records: bytes, world: int, rank: int) -> None:
    """Validates the rank-ordered gather records of `world` ranks on the host
    alone (nd_attn_gather_check); raises NdAttnError when they do not fit."""
    buf = np.frombuffer(records, dtype=np.uint8).copy()
    if buf.size != world * GATHER_BLOB_BYTES:
        raise NdAttnError(ERR_ARG, f"{buf.size} bytes of records for {world} ranks")
    _check(load().nd_attn_gather_check(buf.ctypes.data, world, rank))


def _check(rc: int) -> int:
    if rc < 0:
        raise NdAttnError(rc, load().nd_attn_last_error().decode())
    return rc


def _ptr(x) -> int | None:
    """Device address of a torch CUDA tensor (contiguous), an int, or None."""
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if hasattr(x, "data_ptr"):
        if not x.is_cuda:
            raise ValueError("device entry points take CUDA tensors; use the *_host forms for host arrays")
        if not x.is_contiguous():
            raise ValueError("tensors must be contiguous")
        return x.data_ptr()
    raise TypeError(f"cannot take a device pointer of {type(x)}")


def _hptr(a) -> int | None:
    if a is None:
        return None
    if not isinstance(a, np.ndarray) or not a.flags["C_CONTIGUOUS"]:
        raise ValueError("host entry points take C-contiguous numpy arrays")
    return a.ctypes.data


def _u32(a) -> np.ndarray | None:
    return None if a is None else np.ascontiguousarray(np.asarray(a, dtype=np.uint32))


class Prefix:
    """A saved schema prefix (nd_model_prefix_save's nd_prefix)."""

    def __init__(self, ptr: int, owner: "Attn"):
        self.ptr, self.owner = ptr, owner

    def read(self) -> tuple[np.ndarray, int, int]:
        n, pos, sink = c_size_t(), c_uint32(), c_uint32()
        lib = load()
        _check(lib.nd_attn_prefix_read(self.ptr, None, 0, ctypes.byref(n), ctypes.byref(pos), ctypes.byref(sink)))
        img = np.zeros(n.value, dtype=np.uint8)
        _check(lib.nd_attn_prefix_read(self.ptr, img.ctypes.data, n.value, None, None, None))
        return img, pos.value, sink.value

    def free(self) -> None:
        if self.ptr:
            load().nd_attn_prefix_free(self.ptr)
            self.ptr = 0

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class Attn:
    """One nd_attn handle: caches, session state and the hot path on one GPU."""

    def __init__(self, n_layers=1, n_heads=8, n_kv_heads=8, qk_head_dim=64, v_head_dim=64, window=384,
                 max_seqs=1, block_size=0, n_blocks=0, max_pos=0, rope_theta=10000.0, kv_dtype="f32",
                 act_dtype="f32", out_dtype=None, device=0, qkv_conv_taps=0):
        lib = load()
        cfg = Config()
        lib.nd_attn_config_init(ctypes.byref(cfg))
        dt = lambda d: DT_NAMES[d] if isinstance(d, str) else int(d)  # noqa: E731
        for k, v in dict(n_layers=n_layers, n_heads=n_heads, n_kv_heads=n_kv_heads, qk_head_dim=qk_head_dim,
                         v_head_dim=v_head_dim, window=window, max_seqs=max_seqs, block_size=block_size,
                         n_blocks=n_blocks, max_pos=max_pos or window, rope_theta=rope_theta,
                         kv_dtype=dt(kv_dtype), act_dtype=dt(act_dtype),
                         out_dtype=dt(out_dtype if out_dtype is not None else act_dtype),
                         device=device, qkv_conv_taps=qkv_conv_taps).items():
            setattr(cfg, k, v)
        self.cfg = cfg
        h = c_void_p()
        _check(lib.nd_attn_open(ctypes.byref(cfg), ctypes.byref(h)))
        self.h = h.value
        self.rep = n_heads // n_kv_heads

    # ---- lifetime
    def close(self) -> None:
        if getattr(self, "h", None):
            load().nd_attn_close(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- session state
    def set_head_norm(self, layer: int, q_scale=None, k_scale=None) -> None:
        q = None if q_scale is None else np.ascontiguousarray(q_scale, dtype=np.float32)
        k = None if k_scale is None else np.ascontiguousarray(k_scale, dtype=np.float32)
        _check(load().nd_attn_set_head_norm(self.h, layer, _hptr(q), _hptr(k)))

    def set_conv_taps(self, layer: int, wq, wk, wv) -> None:
        """Tap weights [taps][dim] of the layer's q, k and v projections."""
        w = [np.ascontiguousarray(x, dtype=np.float32) for x in (wq, wk, wv)]
        _check(load().nd_attn_set_conv_taps(self.h, layer, *(_hptr(x) for x in w)))

    def reset(self, seq: int = 0) -> None:
        _check(load().nd_attn_reset(self.h, seq))

    def set_sink(self, seq: int, n: int) -> None:
        _check(load().nd_attn_set_sink(self.h, seq, n))

    def snapshot(self, seq: int = 0) -> None:
        _check(load().nd_attn_snapshot(self.h, seq))

    def rewind(self, seq: int = 0) -> None:
        _check(load().nd_attn_rewind(self.h, seq))

    def advance(self, n: int, seq_ids=None, lens=None) -> None:
        ids, ln = _u32(seq_ids), _u32(lens)
        _check(load().nd_attn_advance(self.h, n, _hptr(ids), _hptr(ln)))

    def state(self, seq: int = 0) -> tuple[int, int]:
        pos, sink = c_uint32(), c_uint32()
        _check(load().nd_attn_get_state(self.h, seq, ctypes.byref(pos), ctypes.byref(sink)))
        return pos.value, sink.value

    def set_state(self, seq: int, pos: int, n_sink: int = 0) -> None:
        _check(load().nd_attn_set_state(self.h, seq, pos, n_sink))

    # ---- hot path (device tensors)
    def decode(self, layer, n, q, k, v, out, gate=None, seq_ids=None) -> None:
        ids = _u32(seq_ids)
        _check(load().nd_attn_decode(self.h, layer, n, _hptr(ids), _ptr(q), _ptr(k), _ptr(v), _ptr(gate),
                                     _ptr(out)))

    def decode_shared(self, layer, n, prefix_seq, prefix_rows, q, k, v, out, gate=None, seq_ids=None) -> None:
        """nd_attn_decode for sequences whose cache rows [0, prefix_rows) equal
        those of prefix_seq (nd_attn_decode_shared): the prefix is read once per
        CTA and shared across the requests."""
        ids = _u32(seq_ids)
        _check(load().nd_attn_decode_shared(self.h, layer, n, _hptr(ids), prefix_seq, prefix_rows, _ptr(q), _ptr(k),
                                            _ptr(v), _ptr(gate), _ptr(out)))

    def prefill(self, layer, lens, q, k, v, out, gate=None, seq_ids=None) -> None:
        ln, ids = _u32(lens), _u32(seq_ids)
        _check(load().nd_attn_prefill(self.h, layer, len(ln), _hptr(ids), _hptr(ln), _ptr(q), _ptr(k), _ptr(v),
                                      _ptr(gate), _ptr(out)))

    def rope_append(self, layer, lens, q, k, v, seq_ids=None) -> None:
        """K1 alone (nd_attn_rope_append): norm + RoPE + KV store of k/v at the
        sequences' current positions; q (or None) rotated in place."""
        ln, ids = _u32(lens), _u32(seq_ids)
        _check(load().nd_attn_rope_append(self.h, layer, len(ln), _hptr(ids), _hptr(ln), _ptr(q), _ptr(k), _ptr(v)))

    def decode_noalloc(self, layer, n, q, k, v, out, gate=None) -> None:
        """nd_attn_decode for sequences 0..n-1 with its scratch in the library's
        fixed device array (no device allocation by the call)."""
        _check(load().nd_attn_decode_noalloc(self.h, layer, n, _ptr(q), _ptr(k), _ptr(v), _ptr(gate), _ptr(out)))

    # ---- head-sharded decode (one rank per GPU)
    def gather_init(self, rank: int, world: int) -> bytes:
        """Allocates this rank's gather buffer; returns the record the other
        ranks need (nd_attn_gather_init)."""
        rec = np.zeros(GATHER_BLOB_BYTES, dtype=np.uint8)
        _check(load().nd_attn_gather_init(self.h, rank, world, rec.ctypes.data))
        return rec.tobytes()

    def gather_attach(self, records: bytes) -> None:
        """Maps the other ranks' buffers from the records of all ranks, in rank
        order (nd_attn_gather_attach)."""
        buf = np.frombuffer(records, dtype=np.uint8).copy()
        _check(load().nd_attn_gather_attach(self.h, buf.ctypes.data))

    def decode_gather(self, layer, n, q, k, v, out, gate=None, seq_ids=None) -> None:
        """nd_attn_decode over this rank's heads, with every rank's heads
        gathered into out [n, world * n_heads * v_head_dim]."""
        ids = _u32(seq_ids)
        _check(load().nd_attn_decode_gather(self.h, layer, n, _hptr(ids), _ptr(q), _ptr(k), _ptr(v), _ptr(gate),
                                            _ptr(out)))

    # ---- hot path (host arrays)
    def decode_host(self, layer, n, q, k, v, out, gate=None, seq_ids=None) -> None:
        ids = _u32(seq_ids)
        _check(load().nd_attn_decode_host(self.h, layer, n, _hptr(ids), _hptr(q), _hptr(k), _hptr(v),
                                          _hptr(gate), _hptr(out)))

    def prefill_host(self, layer, lens, q, k, v, out, gate=None, seq_ids=None) -> None:
        ln, ids = _u32(lens), _u32(seq_ids)
        _check(load().nd_attn_prefill_host(self.h, layer, len(ln), _hptr(ids), _hptr(ln), _hptr(q), _hptr(k),
                                           _hptr(v), _hptr(gate), _hptr(out)))

    # ---- prefix
    def prefix_save(self, seq: int = 0) -> Prefix | None:
        p = load().nd_attn_prefix_save(self.h, seq)
        return Prefix(p, self) if p else None

    def prefix_restore(self, seq: int, prefix: Prefix) -> None:
        _check(load().nd_attn_prefix_restore(self.h, seq, prefix.ptr if prefix else None))

    # ---- cache access
    def read_cache(self, layer: int, seq: int, slot0: int, n: int):
        c = self.cfg
        npdt = {DT_I8: np.int8, DT_F32: np.float32, DT_F16: np.float16, DT_BF16: np.uint16}[c.kv_dtype]
        k = np.zeros((n, c.n_kv_heads * c.qk_head_dim), dtype=npdt)
        v = np.zeros((n, c.n_kv_heads * c.v_head_dim), dtype=npdt)
        ks = vs = None
        if c.kv_dtype == DT_I8:
            ks = np.zeros((n, c.n_kv_heads), dtype=np.float32)
            vs = np.zeros((n, c.n_kv_heads), dtype=np.float32)
        _check(load().nd_attn_read_cache(self.h, layer, seq, slot0, n, _hptr(k), _hptr(v), _hptr(ks), _hptr(vs)))
        return k, v, ks, vs

    def write_cache(self, layer, seq, slot0, n, k, v, k_scale=None, v_scale=None) -> None:
        _check(load().nd_attn_write_cache(self.h, layer, seq, slot0, n, _ptr(k), _ptr(v), _ptr(k_scale),
                                          _ptr(v_scale)))

    def set_block_table(self, seq: int, pages) -> None:
        p = np.ascontiguousarray(np.asarray(pages, dtype=np.int32))
        _check(load().nd_attn_set_block_table(self.h, seq, p.ctypes.data))

    # ---- misc
    def sync(self) -> None:
        _check(load().nd_attn_sync(self.h))

    def selftest_wait(self, limit_us: int = 1000) -> int:
        """Runs the bounded-wait self-test; returns its status code
        (ERR_TIMEOUT when the device status path works)."""
        return load().nd_attn_selftest_wait(self.h, limit_us)

    @property
    def stream(self) -> int:
        return load().nd_attn_stream(self.h) or 0

    def set_stream(self, stream: int | None) -> None:
        _check(load().nd_attn_set_stream(self.h, stream))

    @property
    def launches(self) -> int:
        return load().nd_attn_launch_count(self.h)


class CQ:
    """A `.cact` archive through nd_cq_open (include/nd_cq.h): its header and
    directory, FP16 tensors as floats, and the CQ2 projections on the device
    (device < 0 opens it for reading only)."""

    def __init__(self, blob: bytes, device: int = 0):
        self._buf = ctypes.create_string_buffer(bytes(blob), len(blob))
        h = c_void_p()
        _check(load().nd_cq_open(self._buf, len(blob), device, ctypes.byref(h)))
        self.h = h

    def close(self) -> None:
        if self.h:
            load().nd_cq_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def header(self) -> np.ndarray:
        w = np.zeros(49, np.uint32)
        _check(load().nd_cq_header(self.h, w.ctypes.data))
        return w

    def tensor(self, index: int) -> CqTensor:
        t = CqTensor()
        _check(load().nd_cq_tensor_info(self.h, index, ctypes.byref(t)))
        return t

    def layer_tensor(self, layer: int, slot) -> int:
        i = c_uint32()
        sl = CQ_SLOTS.index(slot) if isinstance(slot, str) else slot
        _check(load().nd_cq_layer_tensor(self.h, layer, sl, ctypes.byref(i)))
        return i.value

    def read_f32(self, index: int) -> np.ndarray:
        t = self.tensor(index)
        n = t.nbytes // (2 if t.dtype == 1 else 4)
        out = np.zeros(max(n, 1), np.float32)
        _check(load().nd_cq_read_f32(self.h, index, out.ctypes.data, out.size))
        return out[:n]

    def project(self, tensors, n_tok: int, x, ys, stream=None) -> None:
        """ys[i] = W_i x for CQ2 tensors reducing over one input (device
        tensors: x [n_tok][in] f32, ys[i] [n_tok][out_i] f32)."""
        ids = np.ascontiguousarray(np.asarray(tensors, dtype=np.uint32))
        outs = (c_void_p * len(ys))(*[_ptr(y) for y in ys])
        _check(load().nd_cq_project(self.h, len(ids), ids.ctypes.data, n_tok, _ptr(x), outs, stream))
