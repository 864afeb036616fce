"""The drop-in boundary without a GPU: libndattn.so loads, exports every entry
point include/nd_attn.h declares, the ctypes view of nd_attn_config matches
the C layout, and opening a handle on a machine without an sm_100 device fails
loudly with ND_ATTN_ERR_NOGPU instead of falling back to anything."""
import ctypes
import os
import subprocess

import numpy as np
import pytest

import ndattn
import ndoracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_exports_every_declared_symbol():
    lib = ndattn.load()
    names = ndattn.header_functions()
    assert len(names) >= 25
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    out = subprocess.run(["nm", "-D", "--defined-only", ndattn.LIB_PATH], capture_output=True, text=True).stdout
    exported = {l.split()[-1] for l in out.splitlines() if " T " in l}
    assert set(names) <= exported
    # nothing but the C ABI leaks out of the library
    assert {n for n in exported if n.startswith("nd")} == set(names)


def test_config_layout_matches_c(tmp_path):
    src = tmp_path / "layout.c"
    fields = [f for f, _ in ndattn.Config._fields_]
    body = "\n".join(f'printf("%zu ", offsetof(nd_attn_config, {f}));' for f in fields)
    src.write_text('#include <stdio.h>\n#include <stddef.h>\n#include "nd_attn.h"\nint main(void){'
                   + body + 'printf("%zu\\n", sizeof(nd_attn_config)); return 0;}\n')
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"), str(src),
                    "-o", str(exe)], check=True)
    got = [int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True).stdout.split()]
    want = [getattr(ndattn.Config, f).offset for f in fields] + [ctypes.sizeof(ndattn.Config)]
    assert got == want


def test_header_compiles_as_cplusplus(tmp_path):
    src = tmp_path / "h.cc"
    src.write_text('#include "nd_attn.h"\nint main(){ nd_attn_config c; nd_attn_config_init(&c); return 0; }\n')
    subprocess.run(["g++", "-std=c++17", "-Wall", "-Werror", "-fsyntax-only", "-I",
                    os.path.join(ROOT, "include"), str(src)], check=True)


def test_config_defaults_and_version():
    lib = ndattn.load()
    cfg = ndattn.Config()
    lib.nd_attn_config_init(ctypes.byref(cfg))
    assert (cfg.n_heads, cfg.n_kv_heads, cfg.qk_head_dim, cfg.v_head_dim) == (8, 8, 64, 64)
    assert cfg.kv_dtype == ndattn.DT_F32 and cfg.rope_theta == 10000.0
    assert b"sm_100a" in lib.nd_attn_version()


def test_open_fails_loudly_without_gpu(has_gpu):
    if has_gpu:
        pytest.skip("a GPU is present")
    with pytest.raises(ndattn.NdAttnError) as e:
        ndattn.Attn()
    assert e.value.code in (ndattn.ERR_NOGPU, ndattn.ERR_CUDA)


def test_geometry_errors_before_any_device_work():
    for kw in (dict(qk_head_dim=80, v_head_dim=80), dict(n_heads=12, n_kv_heads=5),
               dict(n_heads=16, n_kv_heads=1), dict(block_size=48, window=384)):
        with pytest.raises(ndattn.NdAttnError) as e:
            ndattn.Attn(**kw)
        assert e.value.code == ndattn.ERR_GEOM


def test_null_handle_calls_are_rejected():
    lib = ndattn.load()
    assert lib.nd_attn_reset(None, 0) == ndattn.ERR_ARG
    assert lib.nd_attn_sync(None) == ndattn.ERR_ARG
    assert lib.nd_attn_prefix_save(None, 0) is None
    assert lib.nd_attn_prefix_restore(None, 0, None) == ndattn.ERR_ARG
    assert b"handle" in lib.nd_attn_last_error()


def test_oracle_half_conversions_match_numpy():
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(20000).astype(np.float32) * s for s in (1e-8, 1e-5, 1.0, 1e4)]
                       + [np.array([0.0, -0.0, 65504.0, 65519.9, 65520.0, 1e9, -1e9, 5.96e-8, 2.98e-8, 2.99e-8,
                                    6.1e-5, np.inf, -np.inf], np.float32)])
    o = O.orc()
    f16 = np.array([o.ndo_f32_to_f16(float(v)) for v in x], np.uint16)
    assert np.array_equal(f16, x.astype(np.float16).view(np.uint16))
    bf = np.array([o.ndo_f32_to_bf16(float(v)) for v in x], np.uint16)
    assert np.array_equal(bf, O.to_bf16_bits(x))
    back = np.array([o.ndo_f16_to_f32(int(b)) for b in f16], np.float32)
    assert np.array_equal(back, f16.view(np.float16).astype(np.float32))


def test_hook_table_points_at_the_entry_points(tmp_path):
    """nd_attn_cuda_ops() (the engine's swap-in hook, nd_quant.h:229-230 pattern)
    returns a table whose every member is the exported entry point of the same
    name; built as a C program against the header and linked to the library."""
    members = ["open", "close", "set_head_norm", "reset", "set_sink", "snapshot", "rewind", "advance", "decode",
               "prefill", "decode_host", "prefill_host", "prefix_save", "prefix_restore", "prefix_free", "sync",
               "last_error", "set_conv_taps"]
    checks = "\n".join(f'    bad += (void *)o->{m} != (void *)nd_attn_{m};' for m in members)
    src = tmp_path / "ops.c"
    src.write_text('#include <stdio.h>\n#include "nd_attn.h"\nint main(void){\n'
                   '    const nd_attn_ops *o = nd_attn_cuda_ops(); int bad = o->version != ND_ATTN_OPS_VERSION;\n'
                   + checks + '\n    printf("%d\\n", bad); return bad;\n}\n')
    exe = tmp_path / "ops"
    libdir = os.path.dirname(ndattn.LIB_PATH)
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-Wno-pedantic", "-I", os.path.join(ROOT, "include"),
                    str(src), "-o", str(exe), "-L", libdir, "-lndattn", f"-Wl,-rpath,{libdir}"], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True)
    assert r.returncode == 0 and r.stdout.strip() == "0", (r.returncode, r.stdout, r.stderr)
