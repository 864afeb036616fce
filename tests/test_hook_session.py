"""The reference engine with the library behind its attention() seam.

oracle/nd_attn_hook.patch adds the hook INTEGRATION describes (nd_attn_hook,
called after the QKV taps in attention(), engine/src/nd_model.c:2382-2502);
oracle/Makefile applies it to a copy of the reference sources and builds
oracle/_ref/hook_session (oracle/hook_session.c), a gcc-built C program that
runs one sequence of a synthetic archive's layer 0 through attention() twice
per position: on the stock C path, and with the hook calling
nd_attn_decode_host through nd_attn_cuda_ops() from a dlopen'ed
libndattn.so. It checks the library's int8 K/V bytes and scales bit for bit
against the C caches and every output within 1e-3.
"""
import os
import subprocess
import sys

import pytest

import ndattn

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
import make_cact as MC  # noqa: E402

EXE = os.path.join(HERE, "..", "oracle", "_ref", "hook_session")

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("tokens,window,n_sink", [(48, 384, 0), (200, 128, 16)])
def test_patched_engine_through_the_hook(tmp_path, tokens, window, n_sink):
    assert os.path.exists(EXE), "oracle/_ref/hook_session is built by `make -C oracle hook`"
    blob, _ = MC.synthetic_cact(seed=12)
    path = tmp_path / "synthetic.cact"
    path.write_bytes(blob)
    r = subprocess.run([EXE, str(path), ndattn.LIB_PATH, str(tokens), str(window), str(n_sink)],
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and "PASS" in r.stdout, (r.returncode, r.stdout, r.stderr)
