"""The `.cact` reader and the CQ2 projections (include/nd_cq.h), and the whole
attention block of one synthetic-archive layer end to end.

The archive comes from tests/golden/make_cact.py (the reference's format, the
reference model's attention geometry: 12 q / 2 kv heads, qk 48, v 64, d_model
768, 3 QKV taps, theta 1e5, window 384, CQ2 group 128).

CPU (no GPU):
- nd_cq_open parses it as the reference's nd_cact_open does (header words,
  directory records, FP16 tensors as nd_f16 floats) and refuses broken
  archives with nd_cact_open's codes (-1 short, -2 tag, -3 geometry,
  -4 directory past the end, -5 codebook under 28 entries).
- Oracle pin: the reference's own CQ2 projection (nd_cq_prepare + pair table
  + lut2 row walk, oracle/_ref) equals the dequantised-weight restatement
  y = sum_g norm * (H cb[idx]) / sqrt(g) . x_g within f32 rounding.
GPU:
- nd_cq_project equals the reference's projection bit for bit, for every
  projection of the layer and a batch of tokens.
- One layer of the reference's attention() (oracle/_ref, ndref_attention_layer:
  CQ2 q/k/v/gate, taps, norm + RoPE, int8 KV store, attn_heads, gate, CQ2
  out) against nd_cq_project -> nd_attn_decode (taps, norm, RoPE, int8
  append, attention, gate) -> nd_cq_project, token by token: int8 K/V bytes
  and scales bit-exact, outputs within TOL.
"""
import os
import struct
import sys

import numpy as np
import pytest

import ndattn
import ndoracle as O
from harness import TOL, rel_err

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
import make_cact as MC  # noqa: E402

PROJ = ["q_proj", "k_proj", "v_proj", "gate_proj", "out_proj"]


@pytest.fixture(scope="module")
def archive():
    return MC.synthetic_cact(seed=7)


def _hadamard(n):
    h = np.array([[1.0]])
    while h.shape[0] < n:
        h = np.block([[h, h], [h, -h]])
    return h


def test_reader_matches_archive(archive):
    blob, arrays = archive
    c = ndattn.CQ(blob, device=-1)
    hdr = c.header()
    assert list(hdr[:48]) == list(struct.unpack_from("<48I", blob, 0))
    assert hdr[48] == struct.unpack_from("<I", blob, 192)[0]
    assert c.layer_tensor(0, "q_proj") == MC.layer_tensor(0, "q_proj")
    for slot in MC.SLOTS:
        i = c.layer_tensor(0, slot)
        rec = struct.unpack_from("<BBH4IQQII", blob, 196 + 4 * 28 + 44 * i)
        t = c.tensor(i)
        assert (t.dtype, t.ndim) == rec[:2]
        assert list(t.shape)[:t.ndim] == list(rec[3:3 + t.ndim]) and all(v == 0 for v in list(t.shape)[t.ndim:])
        assert (t.offset, t.nbytes, t.group, t.bits) == rec[7:11]
        if t.dtype == 1:
            assert np.array_equal(c.read_f32(i), np.asarray(arrays[f"{slot}.0"], np.float32).reshape(-1))
    with pytest.raises(ndattn.NdAttnError):
        c.layer_tensor(1, 0)
    with pytest.raises(ndattn.NdAttnError) as e:
        c.project([c.layer_tensor(0, "q_proj")], 1, 0, [0])
    assert e.value.code == ndattn.ERR_ARG      # opened without a device
    c.close()


def test_reader_refuses_broken_archives(archive):
    blob, _ = archive
    cases = {-1: blob[:100]}
    bad = bytearray(blob)
    bad[0] ^= 1
    cases[-2] = bytes(bad)
    bad = bytearray(blob)
    struct.pack_into("<I", bad, 4 * 7, 700)           # d_model != heads * v_head_dim
    cases[-3] = bytes(bad)
    bad = bytearray(blob)
    struct.pack_into("<I", bad, 4, 1 << 24)           # directory past the end
    cases[-4] = bytes(bad)
    bad = bytearray(blob)
    struct.pack_into("<I", bad, 8, 20)                # codebook shorter than cb2|cb3|cb4
    cases[-5] = bytes(bad)
    for code, b in cases.items():
        with pytest.raises(ndattn.NdAttnError) as e:
            ndattn.CQ(b, device=-1)
        assert e.value.code == code, (code, e.value)


def test_reference_projection_pins_dequantised_restatement(archive):
    blob, arrays = archive
    rng = np.random.default_rng(8)
    cb = np.frombuffer(blob, "<f4", 4, 196).astype(np.float64)
    for name in PROJ:
        idx, norms = arrays[f"{name}.0"]
        g = 128
        hm = _hadamard(g) / np.sqrt(g)
        w = np.concatenate([(cb[idx[:, i:i + g]] * norms[:, i // g:i // g + 1].astype(np.float64)) @ hm
                            for i in range(0, idx.shape[1], g)], axis=1)
        x = rng.standard_normal(idx.shape[1]).astype(np.float32)
        got = O.ref_cq_project(blob, MC.layer_tensor(0, name), x)
        want = w @ x.astype(np.float64)
        assert np.abs(got - want).max() <= 1e-5 * max(1.0, np.abs(want).max()), name


@pytest.mark.gpu
def test_projection_bit_exact_with_reference(archive):
    import torch
    blob, _ = archive
    c = ndattn.CQ(blob, device=0)
    rng = np.random.default_rng(9)
    n = 5
    for group in (PROJ[:4], PROJ[4:]):
        ids = [c.layer_tensor(0, s) for s in group]
        d_in = c.tensor(ids[0]).shape[1]
        x = (rng.standard_normal((n, d_in)) * rng.uniform(0.1, 3.0, (n, 1))).astype(np.float32)
        x[2, :7] = 0.0
        ys = [torch.full((n, c.tensor(i).shape[0]), float("nan"), device="cuda") for i in ids]
        c.project(ids, n, torch.from_numpy(x).cuda(), ys)
        torch.cuda.synchronize()
        for i, y in zip(ids, ys):
            got = y.cpu().numpy()
            for t in range(n):
                want = O.ref_cq_project(blob, i, x[t])
                assert np.array_equal(got[t].view(np.uint32), want.view(np.uint32)), (i, t)
    c.close()


@pytest.mark.gpu
def test_attention_layer_end_to_end(archive):
    """CQ2 projections -> taps -> norm + RoPE -> int8 KV append -> attention
    -> gate -> CQ2 out projection against the reference's attention()."""
    import torch
    blob, _ = archive
    c = ndattn.CQ(blob, device=0)
    hdr = c.header()
    d_model, H, HKV, QK, VD, taps = (int(hdr[i]) for i in (7, 8, 9, 11, 12, 19))
    theta = struct.unpack("<f", struct.pack("<I", int(hdr[48])))[0]
    W, T = 384, 40
    a = ndattn.Attn(n_layers=1, n_heads=H, n_kv_heads=HKV, qk_head_dim=QK, v_head_dim=VD, window=W,
                    rope_theta=theta, kv_dtype="i8", act_dtype="f32", out_dtype="f32", qkv_conv_taps=taps)
    ids = {s: c.layer_tensor(0, s) for s in MC.SLOTS}
    a.set_head_norm(0, c.read_f32(ids["q_norm"]), c.read_f32(ids["k_norm"]))
    a.set_conv_taps(0, *(c.read_f32(ids[s]).reshape(taps, -1) for s in ("q_taps", "k_taps", "v_taps")))
    ref = O.RefAttentionLayer(blob, W)
    rng = np.random.default_rng(10)
    q = torch.zeros((1, H * QK), device="cuda")
    k = torch.zeros((1, HKV * QK), device="cuda")
    v = torch.zeros((1, HKV * VD), device="cuda")
    gate = torch.zeros((1, H * VD), device="cuda")
    attn = torch.zeros((1, H * VD), device="cuda")
    y = torch.zeros((1, d_model), device="cuda")
    worst = 0.0
    for pos in range(T):
        x = rng.standard_normal(d_model).astype(np.float32)
        want = ref.step(pos, x)
        xd = torch.from_numpy(x).cuda().view(1, -1)
        torch.cuda.synchronize()
        # One stream for the whole block: the projections on the handle's.
        c.project([ids["q_proj"], ids["k_proj"], ids["v_proj"], ids["gate_proj"]], 1, xd, [q, k, v, gate],
                  stream=a.stream)
        a.decode(0, 1, q, k, v, attn, gate=gate)
        c.project([ids["out_proj"]], 1, attn, [y], stream=a.stream)
        a.sync()
        torch.cuda.synchronize()
        worst = max(worst, rel_err(y.cpu().numpy().reshape(-1), want))
        a.advance(1)
    kc, vc, ks, vs = a.read_cache(0, 0, 0, T)
    assert np.array_equal(kc.view(np.int8), ref.k_cache[:T])
    assert np.array_equal(vc.view(np.int8), ref.v_cache[:T])
    assert np.array_equal(ks.view(np.uint32), ref.k_scale[:T].view(np.uint32))
    assert np.array_equal(vs.view(np.uint32), ref.v_scale[:T].view(np.uint32))
    assert worst <= TOL, worst
    a.close()
    c.close()
