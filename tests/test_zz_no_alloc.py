"""nd_attn_decode_noalloc: the decode entry point for callers that may not have
the library allocate device memory after start-up (hosts that hand out every
GPU byte from their own fixed budget, request loops where a cudaMalloc/cudaFree
could synchronise the device or fail). Its split-KV scratch is a fixed array in
the library's device image.

Checked through the C ABI against the regular nd_attn_decode on identical
sessions, two calls in a row (the second call finds the previous call's
contents in the shared array), within the parity tolerance; and the size limit
is refused with a clear error before anything is launched. The file name sorts
last so a run that stops at the first failure has run everything else first;
it also passes alone in a fresh process."""
import numpy as np
import pytest

import ndattn
from harness import TOL, rel_err

pytestmark = pytest.mark.gpu


def _session(ctx, seed):
    import torch
    H = HKV = 8
    a = ndattn.Attn(n_layers=2, n_heads=H, n_kv_heads=HKV, window=2304, max_seqs=len(ctx), kv_dtype="f16",
                    act_dtype="f16", out_dtype="f32", max_pos=2304)
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    for l in range(2):
        for s, n in enumerate(ctx):
            k = (torch.randn((n, HKV * 64), generator=g, device="cuda") * 0.5).half()
            v = (torch.randn((n, HKV * 64), generator=g, device="cuda") * 0.5).half()
            torch.cuda.synchronize()
            a.write_cache(l, s, 0, n, k, v)
    for s, n in enumerate(ctx):
        a.set_state(s, n, 0)
    return a


def test_noalloc_decode_matches_regular_decode_twice():
    import torch
    ctx = [2000, 300, 1500, 64, 1024, 2047, 777, 1]
    reg, fix = _session(ctx, 5), _session(ctx, 5)
    B, H = len(ctx), 8
    g = torch.Generator(device="cuda")
    g.manual_seed(6)
    for call in range(2):
        for l in range(2):
            q = torch.randn((B, H * 64), generator=g, device="cuda").half()
            k = (torch.randn((B, H * 64), generator=g, device="cuda") * 0.5).half()
            v = (torch.randn((B, H * 64), generator=g, device="cuda") * 0.5).half()
            o_reg = torch.zeros((B, H * 64), device="cuda")
            o_fix = torch.full((B, H * 64), float("nan"), device="cuda")
            reg.decode(l, B, q, k, v, o_reg)
            fix.decode_noalloc(l, B, q, k, v, o_fix)
            reg.sync()
            fix.sync()
            assert rel_err(o_fix.cpu().numpy(), o_reg.cpu().numpy()) <= TOL, (call, l)
        reg.advance(B)
        fix.advance(B)
    for l in range(2):
        for s in range(B):
            kr, vr, _, _ = reg.read_cache(l, s, 0, ctx[s] + 2)
            kf, vf, _, _ = fix.read_cache(l, s, 0, ctx[s] + 2)
            assert np.array_equal(kr.view(np.uint16), kf.view(np.uint16))
            assert np.array_equal(vr.view(np.uint16), vf.view(np.uint16))
    reg.close()
    fix.close()


def test_noalloc_rejects_sizes_beyond_the_fixed_scratch():
    import torch
    n = ndattn.NOALLOC_MAX_ITEMS // 8 + 1
    a = ndattn.Attn(n_heads=8, n_kv_heads=8, window=64, max_seqs=n, kv_dtype="f16", act_dtype="f16")
    z = torch.zeros((n, 512), dtype=torch.float16, device="cuda")
    before = a.launches
    with pytest.raises(ndattn.NdAttnError) as e:
        a.decode_noalloc(0, n, z, z, z, z)
    assert e.value.code == ndattn.ERR_RANGE and "exceeds" in str(e.value)
    assert a.launches == before
    a.decode_noalloc(0, n - 1, z, z, z, z)       # at the limit: runs
    a.sync()
    a.close()


@pytest.mark.parametrize("taps", [0, 3])
def test_noalloc_decode_leaves_device_memory_unchanged(taps):
    """The promise itself: after a first call on the device (which looks up
    the array's address and loads the kernels), further calls change the
    device's free memory by nothing, also with QKV conv taps configured (the
    tap buffer was sized at open)."""
    import torch
    H, B = 8, 4
    a = ndattn.Attn(n_layers=1, n_heads=H, n_kv_heads=H, window=512, max_seqs=B, kv_dtype="f16",
                    act_dtype="f16", out_dtype="f32", max_pos=512, qkv_conv_taps=taps)
    if taps:
        r = np.random.default_rng(9)
        a.set_conv_taps(0, *[(r.standard_normal((taps, H * 64)) * 0.5).astype(np.float32) for _ in range(3)])
    for s in range(B):
        a.set_state(s, 100 + 97 * s, 0)
    g = torch.Generator(device="cuda")
    g.manual_seed(7)
    x = [torch.randn((B, H * 64), generator=g, device="cuda").half() for _ in range(3)]
    o = torch.zeros((B, H * 64), device="cuda")
    a.decode_noalloc(0, B, *x, o)                 # first call on the device
    a.sync()
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for _ in range(3):
        a.decode_noalloc(0, B, *x, o)
        a.advance(B)
    a.sync()
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0
    assert torch.isfinite(o).all()
    a.close()


def test_noalloc_fewer_splits_when_partials_exceed_the_array():
    """8000 (sequence, KV head) pairs with one context of 8192 among 999 of 64:
    the split that spreads the rows over the SMs would need more partial slots
    than the fixed array holds, so the call uses fewer splits. The output
    still matches the regular decode (which has its own, larger scratch)."""
    import torch
    H, HD, BS = 8, 64, 64
    n = 1000
    ctx = [64] * (n - 1) + [8192]
    W = 8192 + BS
    nb = W // BS
    # The case reaches the cut: the natural split of this call, computed as the
    # library chooses it (16 CTAs per SM over 148 SMs, splits of whole 64-row
    # iterations), needs more (item, split) slots than the array holds.
    items = n * H
    rows = sum(c + 1 for c in ctx) * H
    chunk = max(-(-rows // (148 * 16)), 128)
    chunk = -(-chunk // 64) * 64
    natural = -(-(max(ctx) + 1) // chunk)
    slots = (8 * 2**20 - ndattn.NOALLOC_MAX_ITEMS * 4 - 256) // ((HD + 2) * 4)
    assert items * natural > slots
    pages_needed = [-(-(c + 2) // BS) for c in ctx]
    n_blocks = sum(pages_needed)
    tables, p0 = [], 0
    for need in pages_needed:
        own = np.arange(p0, p0 + need)
        tables.append(np.concatenate([own, np.full(nb - need, p0)]))
        p0 += need

    def session():
        a = ndattn.Attn(n_layers=1, n_heads=H, n_kv_heads=H, window=W, max_seqs=n, block_size=BS,
                        n_blocks=n_blocks, kv_dtype="f16", act_dtype="f16", out_dtype="f32", max_pos=W)
        g = torch.Generator(device="cuda")
        g.manual_seed(11)
        for s in range(n):
            a.set_block_table(s, tables[s])
            k = (torch.randn((ctx[s], H * HD), generator=g, device="cuda") * 0.5).half()
            v = (torch.randn((ctx[s], H * HD), generator=g, device="cuda") * 0.5).half()
            torch.cuda.synchronize()
            a.write_cache(0, s, 0, ctx[s], k, v)
            a.set_state(s, ctx[s], 0)
        return a

    reg, fix = session(), session()
    g = torch.Generator(device="cuda")
    g.manual_seed(12)
    for call in range(2):
        q = torch.randn((n, H * HD), generator=g, device="cuda").half()
        k = (torch.randn((n, H * HD), generator=g, device="cuda") * 0.5).half()
        v = (torch.randn((n, H * HD), generator=g, device="cuda") * 0.5).half()
        o_reg = torch.zeros((n, H * HD), device="cuda")
        o_fix = torch.full((n, H * HD), float("nan"), device="cuda")
        reg.decode(0, n, q, k, v, o_reg)
        fix.decode_noalloc(0, n, q, k, v, o_fix)
        reg.sync()
        fix.sync()
        assert rel_err(o_fix.cpu().numpy(), o_reg.cpu().numpy()) <= TOL, call
        reg.advance(n)
        fix.advance(n)
    reg.close()
    fix.close()
