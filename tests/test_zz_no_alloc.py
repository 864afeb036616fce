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
