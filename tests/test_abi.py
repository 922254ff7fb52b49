"""The C-ABI library loads and exports every symbol include/ds_cuda.h
declares; host-side logic that needs no GPU."""
import ctypes

import numpy as np

from conftest import HAS_GPU
from ds_ocr_b200 import _lib, synth


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    declared = _lib.declared_symbols()
    assert len(declared) >= 25
    missing = [s for s in declared if not hasattr(lib, s)]
    assert not missing, missing
    # and the Python binding covers exactly the declared set
    assert sorted(_lib.SIGNATURES) == declared


def test_init_without_gpu_returns_null():
    lib = _lib.load()
    if HAS_GPU:
        return
    assert not lib.ds_cuda_init(0)
    assert lib.ds_cuda_is_available(None) == 0
    assert b"no context" in lib.ds_cuda_last_error(None)


def test_invalid_context_calls_fail_loudly():
    lib = _lib.load()
    x = np.zeros(1280, np.float32)
    assert lib.ds_cuda_lm_head_argmax(None, x.ctypes.data, x.ctypes.data, 1280, 10) < 0
    assert lib.ds_cuda_moe_experts(None, None, None, None, None, 0, 1280, 896, None) < 0
    assert lib.ds_cuda_set_numerics(None, 0, 0) < 0


def test_synth_is_counter_based():
    a = synth.normal_bf16(100000, 42)
    b = synth.normal_bf16(100000, 42)
    c = np.empty(100000, np.uint16)
    synth.fill_bf16(c[:50000], 42)
    assert np.array_equal(a, b) and np.array_equal(a[:50000], c[:50000])
    f = synth.bf16_to_f32(synth.normal_bf16(1 << 20, 7))
    assert abs(f.mean()) < 1e-4 and abs(f.std() - 0.02) < 2e-4
    e = np.empty(1000, np.float32)
    synth.fill_f32_bf16exact(e, 3)
    assert np.all((e.view(np.uint32) & 0xFFFF) == 0)


def test_widened_entry_points_reject_a_missing_context():
    # sampling, history, uniforms, window, embeddings, prefill, KV readback
    # and checkpoint ingest: a NULL context is an error status, not a crash
    lib = _lib.load()
    x = np.zeros(1280, np.float32)
    t = np.zeros(4, np.int32)
    assert lib.ds_cuda_decoder_set_sampling(None, 1, 1.2, 3, 0.0) < 0
    assert lib.ds_cuda_decoder_set_history(None, 1, t.ctypes.data, 4) < 0
    assert lib.ds_cuda_decoder_get_history(None, 1, t.ctypes.data, 4) < 0
    assert lib.ds_cuda_decoder_set_uniforms(None, 1, x.ctypes.data, 4) < 0
    assert lib.ds_cuda_decoder_set_window(None, 1, 8, 16) < 0
    assert lib.ds_cuda_decoder_set_embeddings(None, 1, x.ctypes.data) < 0
    assert lib.ds_cuda_decoder_prefill(None, 1, x.ctypes.data, 1, None, None) < 0
    assert lib.ds_cuda_decoder_prefill_dev(None, 1, x.ctypes.data, 1, None) < 0
    assert lib.ds_cuda_decoder_get_kv(None, 1, 0, 0, 1, x.ctypes.data, x.ctypes.data) < 0
    assert lib.ds_cuda_decoder_create_from_safetensors(None, b"/nonexistent", None) < 0


def test_header_compiles_as_c_and_links(tmp_path):
    # the boundary is a C ABI: a C host includes the header, links the
    # library and gets error statuses (not crashes) without a device
    import os
    import subprocess
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    src = tmp_path / "host.c"
    src.write_text(
        '#include <stdio.h>\n#include "ds_cuda.h"\n'
        "int main(void) {\n"
        "    ds_cuda_ctx_t *c = ds_cuda_init(0);\n"
        "    ds_cuda_decoder_config_t cfg = {0};\n"
        "    int rc = ds_cuda_decoder_create_from_safetensors(c, \"/nonexistent\", &cfg);\n"
        "    printf(\"%d %d\\n\", c != 0, rc < 0);\n"
        "    if (c) ds_cuda_free(c);\n"
        "    return 0;\n"
        "}\n")
    lib_dir = os.path.dirname(_lib.LIB_PATH)
    exe = tmp_path / "host"
    r = subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-I", os.path.join(root, "include"), str(src),
                        "-o", str(exe), "-L", lib_dir, "-l:" + os.path.basename(_lib.LIB_PATH),
                        "-Wl,-rpath," + lib_dir], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stderr
    has_ctx, failed = out.stdout.split()
    assert failed == "1"
    if not HAS_GPU:
        assert has_ctx == "0"
