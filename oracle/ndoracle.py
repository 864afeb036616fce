"""TEST INFRASTRUCTURE ONLY - ctypes view of the CPU checkers in oracle/.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
legs may import this module. It never runs on the product path.

  OracleSeq  one sequence of the restatement (nd_oracle.c), any KV dtype,
             fp64 attention: the tolerance reference.
  RefSeq     one sequence of the reference engine's own C code
             (_ref/libndref.so, built from engine/src/nd_model.c by the
             Makefile here): int8 KV only, the reference's fp32 arithmetic.

Both keep the reference's session rules: kv_slot (nd_model.c:1304-1309),
set_sink's ND_MIN_RECENT cap (1312-1321), snapshot/rewind (1395-1460) and the
saved-prefix image (prefix_copy, 1462-1555).
"""
from __future__ import annotations

import ctypes
import os
import struct
from ctypes import POINTER, c_double, c_float, c_int, c_int32, c_long, c_size_t, c_uint16, c_uint32, c_void_p

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "libndoracle.so")
REF_SO = os.path.join(HERE, "_ref", "libndref.so")

I8, F32, F16, BF16 = 0, 1, 2, 3
NP_KV = {I8: np.int8, F32: np.float32, F16: np.uint16, BF16: np.uint16}


class Geom(ctypes.Structure):
    _fields_ = [("n_heads", c_uint32), ("n_kv_heads", c_uint32), ("qk_head_dim", c_uint32),
                ("v_head_dim", c_uint32), ("window", c_uint32), ("kv_dtype", c_int32)]


class RefGeom(ctypes.Structure):
    _fields_ = [("n_layers", c_uint32), ("n_heads", c_uint32), ("n_kv_heads", c_uint32),
                ("qk_head_dim", c_uint32), ("v_head_dim", c_uint32), ("window", c_uint32)]


_orc = None
_ref = None


def build() -> None:
    """Builds the checkers (make -C oracle); the reference part only where its sources exist."""
    import subprocess
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def orc() -> ctypes.CDLL:
    global _orc
    if _orc is None:
        if not os.path.exists(ORACLE_SO):
            build()
        lib = ctypes.CDLL(ORACLE_SO)
        fp = POINTER(c_float)
        lib.ndo_token.restype = c_int
        lib.ndo_token.argtypes = [POINTER(Geom), c_void_p, c_void_p, c_void_p, c_void_p, c_uint32, c_uint32,
                                  c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                  c_void_p, c_void_p]
        lib.ndo_conv_taps.restype = c_int
        lib.ndo_conv_taps.argtypes = [c_uint32, c_uint32, c_uint32, c_void_p, c_void_p, c_void_p, c_void_p]
        lib.ndo_rope_table.argtypes = [c_float, c_uint32, c_uint32, c_void_p]
        lib.ndo_rope_table.restype = None
        lib.ndo_kv_slot.restype = c_uint32
        lib.ndo_kv_slot.argtypes = [c_uint32, c_uint32, c_uint32]
        lib.ndo_set_sink.restype = c_uint32
        lib.ndo_set_sink.argtypes = [c_uint32, c_uint32]
        lib.ndo_f32_to_f16.restype = c_uint16
        lib.ndo_f32_to_f16.argtypes = [c_float]
        lib.ndo_f16_to_f32.restype = c_float
        lib.ndo_f16_to_f32.argtypes = [c_uint16]
        lib.ndo_f32_to_bf16.restype = c_uint16
        lib.ndo_f32_to_bf16.argtypes = [c_float]
        lib.ndo_bf16_to_f32.restype = c_float
        lib.ndo_bf16_to_f32.argtypes = [c_uint16]
        _ = fp
        _orc = lib
    return _orc


def ref_available() -> bool:
    return os.path.exists(REF_SO)


def ref() -> ctypes.CDLL:
    global _ref
    if _ref is None:
        if not os.path.exists(REF_SO):
            raise FileNotFoundError(f"{REF_SO} missing: built only where the reference sources are present")
        lib = ctypes.CDLL(REF_SO)
        lib.ndref_attn_token.restype = c_int
        lib.ndref_attn_token.argtypes = [POINTER(RefGeom)] + [c_void_p] * 4 + [c_uint32] * 3 + [c_void_p] * 9
        lib.ndref_kv_slot.restype = c_uint32
        lib.ndref_kv_slot.argtypes = [c_uint32, c_uint32, c_uint32]
        lib.ndref_set_sink.restype = c_uint32
        lib.ndref_set_sink.argtypes = [c_uint32, c_uint32]
        lib.ndref_rope_inv.argtypes = [c_float, c_uint32, c_void_p]
        lib.ndref_rope_at.argtypes = [c_void_p, c_uint32, c_uint32, c_void_p, c_void_p]
        lib.ndref_prefix_image.restype = c_long
        lib.ndref_prefix_image.argtypes = [POINTER(RefGeom), c_void_p, c_void_p, c_void_p, c_void_p, c_uint32,
                                           c_uint32, c_void_p, c_void_p, c_void_p, c_void_p, c_size_t,
                                           POINTER(c_uint32)]
        lib.ndref_norm_rope.restype = c_int
        lib.ndref_norm_rope.argtypes = [POINTER(RefGeom), c_void_p, c_uint32, c_void_p, c_void_p, c_void_p]
        lib.ndref_cq_project.restype = c_int
        lib.ndref_cq_project.argtypes = [c_void_p, c_size_t, c_uint32, c_void_p, c_void_p]
        lib.ndref_attention_layer.restype = c_int
        lib.ndref_attention_layer.argtypes = [c_void_p, c_size_t, c_uint32, c_uint32, c_uint32] + [c_void_p] * 11
        lib.ndref_tap.restype = c_int
        lib.ndref_tap.argtypes = [c_uint32, c_uint32, c_uint32, c_void_p, c_void_p, c_void_p]
        lib.ndref_prefill_bench.restype = c_double
        lib.ndref_prefill_bench.argtypes = [POINTER(RefGeom), c_uint32, c_uint32, c_uint32, c_float, c_uint32]
        lib.ndref_decode_bench.restype = c_double
        lib.ndref_decode_bench.argtypes = [POINTER(RefGeom), c_uint32, c_void_p, c_uint32, c_uint32, c_float,
                                           c_uint32]
        _ref = lib
    return _ref


def _p(a):
    return None if a is None else a.ctypes.data


# ------------------------------------------------------------ conversions
def to_f16_bits(x: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(x, dtype=np.float32).astype(np.float16).view(np.uint16)


def to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bits, round to nearest even (NaN kept quiet)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(nan, ((u >> 16) | 0x40).astype(np.uint16), r)


def from_bf16_bits(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_act(x: np.ndarray, dt: int) -> np.ndarray:
    """Values an activation of dtype dt carries, as float32."""
    x = np.asarray(x, dtype=np.float32)
    if dt == F16:
        return x.astype(np.float16).astype(np.float32)
    if dt == BF16:
        return from_bf16_bits(to_bf16_bits(x))
    return x


def rope_table(theta: float, qk: int, npos: int) -> np.ndarray:
    """[npos][qk/2][2] cos/sin with the reference's expressions."""
    tab = np.zeros((npos, qk // 2, 2), dtype=np.float32)
    orc().ndo_rope_table(c_float(theta), qk, npos, tab.ctypes.data)
    return tab


def kv_slot(window: int, n_sink: int, p: int) -> int:
    return int(orc().ndo_kv_slot(window, n_sink, p))


def set_sink_cap(window: int, n: int) -> int:
    return int(orc().ndo_set_sink(window, n))


# ------------------------------------------------------------ sequences
class _SeqBase:
    """One sequence of the reference session. taps > 0 adds the QKV short
    causal convolution ahead of the path (tap_projection, nd_model.c:2361-2379)
    with its per-layer history; act_dtype is the activation type its output is
    rounded to (the GPU path stores convolved rows in that type)."""

    def __init__(self, n_layers, n_heads, n_kv_heads, qk, vd, window, kv_dtype, theta=10000.0, max_pos=None,
                 taps=0, act_dtype=F32):
        self.L, self.H, self.HKV, self.QK, self.VD, self.W = n_layers, n_heads, n_kv_heads, qk, vd, window
        self.kv_dtype = kv_dtype
        npdt = NP_KV[kv_dtype]
        self.k = np.zeros((n_layers, window, n_kv_heads * qk), dtype=npdt)
        self.v = np.zeros((n_layers, window, n_kv_heads * vd), dtype=npdt)
        self.ks = np.zeros((n_layers, window, n_kv_heads), dtype=np.float32)
        self.vs = np.zeros((n_layers, window, n_kv_heads), dtype=np.float32)
        self.pos = self.n_sink = self.snap_pos = 0
        self.has_snap = False
        self.tab = rope_table(theta, qk, max_pos or window)
        self.norms: dict[int, tuple[np.ndarray, np.ndarray]] = {}
        self.T, self.act_dtype = taps, act_dtype
        dims = (n_heads * qk, n_kv_heads * qk, n_kv_heads * vd)
        # q_hist / k_hist / v_hist [layers][taps][dim] and the snapshot copies
        self.hist = [np.zeros((n_layers, taps, d), np.float32) for d in dims]
        self.snap_hist = [h.copy() for h in self.hist]
        ident = [np.zeros((taps, d), np.float32) for d in dims]
        for w in ident:
            w[:1] = 1.0
        self.tapw = {layer: ident for layer in range(n_layers)}

    def set_conv_taps(self, layer, wq, wk, wv):
        self.tapw[layer] = [np.ascontiguousarray(w, dtype=np.float32) for w in (wq, wk, wv)]

    def conv(self, layer, pos, q, k, v):
        """The convolved q, k, v of the token at `pos` (history updated)."""
        out = []
        for x, w, h in zip((q, k, v), self.tapw[layer], self.hist):
            x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
            hl = np.ascontiguousarray(h[layer])
            y = np.zeros_like(x)
            assert orc().ndo_conv_taps(self.T, pos, x.size, w.ctypes.data, x.ctypes.data, hl.ctypes.data,
                                       y.ctypes.data) == 0
            h[layer] = hl
            out.append(round_act(y, self.act_dtype))
        return out

    # reference session rules
    def reset(self):
        self.pos = self.n_sink = 0
        self.has_snap = False
        for h in self.hist:
            h[...] = 0.0

    def set_sink(self, n):
        self.n_sink = set_sink_cap(self.W, n)

    def snapshot(self):
        self.set_sink(self.pos)
        self.snap_pos = self.pos
        self.has_snap = True
        self.snap_hist = [h.copy() for h in self.hist]

    def rewind(self):
        if not self.has_snap:
            self.reset()
        else:
            self.pos = self.snap_pos
            self.hist = [h.copy() for h in self.snap_hist]

    def advance(self, n=1):
        self.pos += n

    def prefix_image(self) -> bytes:
        """prefix_copy's byte order (nd_model.c:1493-1529): K live rows per
        layer, then V, then the int8 scales."""
        live = min(self.snap_pos + 1, self.W)
        parts = [self.k[:, :live], self.v[:, :live]]
        if self.kv_dtype == I8:
            parts += [self.ks[:, :live], self.vs[:, :live]]
        parts += self.snap_hist          # q_hist, k_hist, v_hist of the snapshot (empty without taps)
        return b"".join(np.ascontiguousarray(p).tobytes() for p in parts)

    def prefix_save(self):
        if not self.has_snap or self.pos != self.snap_pos:
            return None
        live = min(self.snap_pos + 1, self.W)
        return dict(pos=self.snap_pos, sink=self.n_sink, live=live, k=self.k[:, :live].copy(),
                    v=self.v[:, :live].copy(), ks=self.ks[:, :live].copy(), vs=self.vs[:, :live].copy(),
                    hist=[h.copy() for h in self.snap_hist])

    def prefix_restore(self, p):
        self.snap_pos, self.n_sink = p["pos"], p["sink"]
        live = p["live"]
        self.k[:, :live], self.v[:, :live] = p["k"], p["v"]
        self.ks[:, :live], self.vs[:, :live] = p["ks"], p["vs"]
        self.snap_hist = [h.copy() for h in p["hist"]]
        self.has_snap = True
        self.rewind()

    def cs_sn(self, pos):
        t = self.tab[pos]
        return np.ascontiguousarray(t[:, 0]), np.ascontiguousarray(t[:, 1])


class OracleSeq(_SeqBase):
    """The restatement; step() returns float64 [n_heads][v_hd]."""

    def step(self, layer, q, k, v, gate=None, off=0):
        pos = self.pos + off
        if self.T:
            q, k, v = self.conv(layer, pos, q, k, v)
        g = Geom(self.H, self.HKV, self.QK, self.VD, self.W, self.kv_dtype)
        q = np.array(q, dtype=np.float32, copy=True).reshape(-1)
        k = np.array(k, dtype=np.float32, copy=True).reshape(-1)
        v = np.ascontiguousarray(v, dtype=np.float32).reshape(-1)
        gt = None if gate is None else np.ascontiguousarray(gate, dtype=np.float32).reshape(-1)
        out = np.zeros(self.H * self.VD, dtype=np.float64)
        cs, sn = self.cs_sn(pos)
        qn, kn = self.norms.get(layer, (None, None))
        rc = orc().ndo_token(ctypes.byref(g), self.k[layer].ctypes.data, self.v[layer].ctypes.data,
                             self.ks[layer].ctypes.data, self.vs[layer].ctypes.data, pos, self.n_sink,
                             cs.ctypes.data, sn.ctypes.data, _p(qn), _p(kn), q.ctypes.data, k.ctypes.data,
                             v.ctypes.data, _p(gt), out.ctypes.data)
        assert rc == 0
        return out.reshape(self.H, self.VD)


class RefSeq(_SeqBase):
    """The reference engine's own attention (int8 KV); step() returns float32."""

    def __init__(self, *a, **kw):
        super().__init__(*a, **kw)
        assert self.kv_dtype == I8

    def geom(self):
        return RefGeom(self.L, self.H, self.HKV, self.QK, self.VD, self.W)

    def conv(self, layer, pos, q, k, v):
        """The reference's own tap_projection on q, k, v (history updated)."""
        out = []
        for x, w, h in zip((q, k, v), self.tapw[layer], self.hist):
            y = np.array(x, dtype=np.float32, copy=True).reshape(-1)
            hl = np.ascontiguousarray(h[layer])
            assert ref().ndref_tap(self.T, pos, y.size, w.ctypes.data, y.ctypes.data, hl.ctypes.data) == 0
            h[layer] = hl
            out.append(y)
        return out

    def step(self, layer, q, k, v, gate=None, off=0):
        pos = self.pos + off
        if self.T:
            q, k, v = self.conv(layer, pos, q, k, v)
        g = self.geom()
        q = np.array(q, dtype=np.float32, copy=True).reshape(-1)
        k = np.array(k, dtype=np.float32, copy=True).reshape(-1)
        v = np.ascontiguousarray(v, dtype=np.float32).reshape(-1)
        gt = None if gate is None else np.ascontiguousarray(gate, dtype=np.float32).reshape(-1)
        out = np.zeros(self.H * self.VD, dtype=np.float32)
        cs, sn = self.cs_sn(pos)
        qn, kn = self.norms.get(layer, (None, None))
        rc = ref().ndref_attn_token(ctypes.byref(g), self.k.ctypes.data, self.v.ctypes.data, self.ks.ctypes.data,
                                    self.vs.ctypes.data, layer, pos, self.n_sink, cs.ctypes.data, sn.ctypes.data,
                                    _p(qn), _p(kn), q.ctypes.data, k.ctypes.data, v.ctypes.data, _p(gt),
                                    out.ctypes.data)
        assert rc == 0
        return out.reshape(self.H, self.VD)

    def ref_prefix_image(self) -> tuple[bytes, int]:
        """The image the reference's own nd_model_snapshot + prefix_save make at pos."""
        g = self.geom()
        sink = c_uint32()
        hist = [np.ascontiguousarray(h) for h in self.hist]
        hp = [h.ctypes.data if self.T else None for h in hist]
        n = ref().ndref_prefix_image(ctypes.byref(g), self.k.ctypes.data, self.v.ctypes.data, self.ks.ctypes.data,
                                     self.vs.ctypes.data, self.pos, self.T, *hp, None, 0, ctypes.byref(sink))
        buf = np.zeros(max(n, 1), dtype=np.uint8)
        ref().ndref_prefix_image(ctypes.byref(g), self.k.ctypes.data, self.v.ctypes.data, self.ks.ctypes.data,
                                 self.vs.ctypes.data, self.pos, self.T, *hp, buf.ctypes.data, buf.size,
                                 ctypes.byref(sink))
        return buf[:n].tobytes(), sink.value


def ref_norm_rope(x, n_heads, qk, theta, pos, norm=None):
    """Rows x [n_heads * qk] after the reference's own zcrms_heads (with
    `norm`) or apply_rope (without) at `pos`."""
    y = np.array(x, dtype=np.float32, copy=True).reshape(-1)
    cs, sn = ref_rope(theta, qk, pos)
    g = RefGeom(1, n_heads, n_heads, qk, qk, max(pos + 1, 2))
    nm = None if norm is None else np.ascontiguousarray(norm, dtype=np.float32)
    assert ref().ndref_norm_rope(ctypes.byref(g), y.ctypes.data, n_heads, _p(nm), cs.ctypes.data, sn.ctypes.data) == 0
    return y


def ref_cq_project(blob: bytes, index: int, x):
    """W x for CQ2 tensor `index` of a .cact archive through the reference's
    own nd_cq_prepare + nd_cq_lut_build + nd_cq_gemv_lut2 (nd_quant.c)."""
    buf = ctypes.create_string_buffer(blob, len(blob))
    out_rows = struct.unpack_from("<I", blob, _cact_record(blob, index) + 4)[0]
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.zeros(out_rows, np.float32)
    assert ref().ndref_cq_project(buf, len(blob), index, x.ctypes.data, y.ctypes.data) == 0
    return y


def _cact_record(blob: bytes, index: int) -> int:
    """Byte offset of directory record `index` (nd_cact.c: header 196 B, then the codebook)."""
    cb_len = struct.unpack_from("<I", blob, 8)[0]
    return 196 + 4 * cb_len + 44 * index


class RefAttentionLayer:
    """The reference's whole attention() on layer 0 of a .cact archive, one
    token per call (ndref_attention_layer): owns the int8 caches, scales and
    QKV tap histories of one sequence."""

    def __init__(self, blob: bytes, window: int, n_sink: int = 0):
        h = struct.unpack_from("<48If", blob, 0)
        self.blob = ctypes.create_string_buffer(blob, len(blob))
        self.size = len(blob)
        (self.d_model, self.n_heads, self.n_kv, self.qk, self.vd) = h[7], h[8], h[9], h[11], h[12]
        self.taps, self.theta = h[19], h[48]
        self.window, self.n_sink = window, n_sink
        self.k_cache = np.zeros((window, self.n_kv * self.qk), np.int8)
        self.v_cache = np.zeros((window, self.n_kv * self.vd), np.int8)
        self.k_scale = np.zeros((window, self.n_kv), np.float32)
        self.v_scale = np.zeros((window, self.n_kv), np.float32)
        self.q_hist = np.zeros((self.taps, self.n_heads * self.qk), np.float32)
        self.k_hist = np.zeros((self.taps, self.n_kv * self.qk), np.float32)
        self.v_hist = np.zeros((self.taps, self.n_kv * self.vd), np.float32)

    def step(self, pos: int, x):
        cs, sn = ref_rope(self.theta, self.qk, pos)
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.zeros(self.d_model, np.float32)
        arrs = [self.k_cache, self.v_cache, self.k_scale, self.v_scale, cs, sn, self.q_hist, self.k_hist,
                self.v_hist, x, out]
        assert ref().ndref_attention_layer(self.blob, self.size, self.window, pos, self.n_sink,
                                           *[a.ctypes.data for a in arrs]) == 0
        return out


def ref_rope(theta, qk, pos):
    """cos/sin at pos through the reference's own loops."""
    inv = np.zeros(qk // 2, np.float32)
    cs = np.zeros(qk // 2, np.float32)
    sn = np.zeros(qk // 2, np.float32)
    ref().ndref_rope_inv(c_float(theta), qk, inv.ctypes.data)
    ref().ndref_rope_at(inv.ctypes.data, qk, pos, cs.ctypes.data, sn.ctypes.data)
    return cs, sn


def ref_decode_bench(n_heads, n_kv, qk, vd, window, ctx, steps, layers, theta, threads) -> float:
    g = RefGeom(layers, n_heads, n_kv, qk, vd, window)
    c = np.ascontiguousarray(ctx, dtype=np.uint32)
    return float(ref().ndref_decode_bench(ctypes.byref(g), len(c), c.ctypes.data, steps, layers, c_float(theta),
                                          threads))


def ref_prefill_bench(n_heads, n_kv, qk, vd, window, n_seqs, tokens, layers, theta, threads) -> float:
    g = RefGeom(layers, n_heads, n_kv, qk, vd, window)
    return float(ref().ndref_prefill_bench(ctypes.byref(g), n_seqs, tokens, layers, c_float(theta), threads))
