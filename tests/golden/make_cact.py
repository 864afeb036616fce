"""Writes small synthetic `.cact` archives in the reference's format, for the
CQ2 projection and attention-layer parity tests.

Format (engine/include/nd_cact.h:1-99, engine/src/nd_cact.c), little-endian:
  0x00  196-byte header: 49 u32-sized fields in nd_cact_header order
  0xC4  codebook: codebook_len f32 = cb2[4] | cb3[8] | cb4[16]
        directory: num_tensors 44-byte records
        {u8 dtype, u8 ndim, u16 pad, u32 shape[4], u64 offset, u64 nbytes, u32 group, u32 bits}
  ...   tensor blobs, each 64-byte aligned
A CQ tensor [out][in] stores its 2-bit indices as an LSB-first bit stream per
row (in padded to a multiple of `group`), then an f16 norm per (row, group).

Tensor order is the positional layout nd_model_open binds
(engine/src/nd_model.c:642-658, 763-797): tensor 0 the embedding, then per
layer 27 slots (24 without QKV taps): norm_in, q_proj, k_proj, v_proj,
q_taps, k_taps, v_taps, q_norm, k_norm, gate_proj, out_proj, post_norm,
attn_gate, pre_hada, d1, d2, b2, d3, d4, w1a, w1b, w2a, w2b, w3a, w3b,
cond_v, cond_u. Only the attention block's slots carry meaningful values
here; the rest are small f16 placeholders.

Default geometry: the reference model's attention (12 q / 2 kv heads, qk 48,
v 64, d_model 768, window 384, 3 QKV taps, RoPE theta 1e5), CQ2 group 128.

    python tests/golden/make_cact.py out.cact      # writes one archive
"""
import struct
import sys

import numpy as np

TAG = 0x05E12A84
ALIGN = 64
DT_FP16, DT_FP32, DT_CQ = 1, 2, 3
SLOTS = ["norm_in", "q_proj", "k_proj", "v_proj", "q_taps", "k_taps", "v_taps", "q_norm", "k_norm",
         "gate_proj", "out_proj", "post_norm", "attn_gate", "pre_hada", "d1", "d2", "b2", "d3", "d4",
         "w1a", "w1b", "w2a", "w2b", "w3a", "w3b", "cond_v", "cond_u"]


def pack_cq2(idx, norms):
    """[out][in_pad] indices 0..3 -> LSB-first 2-bit rows, then f16 norms [out][ngroup]."""
    out, in_pad = idx.shape
    q = idx.reshape(out, in_pad // 4, 4).astype(np.uint8)
    packed = q[..., 0] | (q[..., 1] << 2) | (q[..., 2] << 4) | (q[..., 3] << 6)
    return packed.tobytes() + norms.astype("<f2").tobytes()


def synthetic_cact(seed=0, d_model=768, n_heads=12, n_kv=2, qk=48, vd=64, window=384, taps=3, group=128,
                   theta=1.0e5, n_layers=1):
    """Returns the archive bytes and a dict of the tensors' source arrays."""
    rng = np.random.default_rng(seed)
    assert n_heads * vd == d_model and n_heads % n_kv == 0 and group % 16 == 0
    q_dim, k_dim, v_dim, attn_dim = n_heads * qk, n_kv * qk, n_kv * vd, n_heads * vd
    cb2 = np.array([-1.5, -0.5, 0.5, 1.5], np.float32) / np.float32(np.sqrt(group))
    cb3 = np.linspace(-1.75, 1.75, 8).astype(np.float32) / np.float32(np.sqrt(group))
    cb4 = np.linspace(-1.875, 1.875, 16).astype(np.float32) / np.float32(np.sqrt(group))
    codebook = np.concatenate([cb2, cb3, cb4]).astype("<f4")

    tensors = []   # (dtype, shape, payload bytes, group, bits)
    arrays = {}

    def f16(name, shape, values):
        arr = np.asarray(values, np.float16).reshape(shape)
        arrays[name] = arr
        tensors.append((DT_FP16, shape, arr.astype("<f2").tobytes(), 0, 16))

    def cq2(name, out, inp):
        in_pad = (inp + group - 1) // group * group
        idx = rng.integers(0, 4, size=(out, in_pad))
        norms = rng.uniform(0.2, 0.4, size=(out, in_pad // group)).astype(np.float16)
        arrays[name] = (idx, norms)
        tensors.append((DT_CQ, (out, inp), pack_cq2(idx, norms), group, 2))

    f16("embedding", (16, d_model), rng.standard_normal((16, d_model)) * 0.1)
    for li in range(n_layers):
        for s in SLOTS:
            name = f"{s}.{li}"
            if s == "q_proj":
                cq2(name, q_dim, d_model)
            elif s == "k_proj":
                cq2(name, k_dim, d_model)
            elif s == "v_proj":
                cq2(name, v_dim, d_model)
            elif s == "gate_proj":
                cq2(name, attn_dim, d_model)
            elif s == "out_proj":
                cq2(name, d_model, attn_dim)
            elif s in ("q_taps", "k_taps", "v_taps"):
                dim = {"q_taps": q_dim, "k_taps": k_dim, "v_taps": v_dim}[s]
                w = np.array([0.7, 0.25, 0.05])[:taps, None] + rng.standard_normal((taps, dim)) * 0.05
                f16(name, (taps, dim), w)
            elif s in ("q_norm", "k_norm"):
                f16(name, (qk,), rng.standard_normal(qk) * 0.1)
            else:
                f16(name, (8,), rng.standard_normal(8) * 0.1)

    n = len(tensors)
    hdr = [TAG, n, len(codebook), window, 8, 16, 16, d_model, n_heads, n_kv, n_layers, qk, vd, window,
           d_model, 1, window, 0, 0, taps, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0] + [0] * 16
    assert len(hdr) == 48
    head = struct.pack("<48I", *hdr) + struct.pack("<f", theta)
    assert len(head) == 196
    dir_off = len(head) + 4 * len(codebook)
    off = (dir_off + 44 * n + ALIGN - 1) // ALIGN * ALIGN
    records, blobs = [], []
    for dt, shape, payload, g, bits in tensors:
        shp = list(shape) + [0] * (4 - len(shape))
        records.append(struct.pack("<BBH4IQQII", dt, len(shape), 0, *shp, off, len(payload), g, bits))
        blobs.append((off, payload))
        off = (off + len(payload) + ALIGN - 1) // ALIGN * ALIGN
    buf = bytearray(off)
    buf[:196] = head
    buf[196:dir_off] = codebook.tobytes()
    buf[dir_off:dir_off + 44 * n] = b"".join(records)
    for o, payload in blobs:
        buf[o:o + len(payload)] = payload
    return bytes(buf), arrays


def layer_tensor(layer, slot, taps=3):
    """Directory index of a layer's slot (nd_model.c:644)."""
    return 1 + layer * (27 if taps else 24) + SLOTS.index(slot)


if __name__ == "__main__":
    blob, _ = synthetic_cact()
    with open(sys.argv[1] if len(sys.argv) > 1 else "synthetic.cact", "wb") as f:
        f.write(blob)
