"""The C-ABI library: loads without a GPU, exports every function the public
header declares, validates arguments before touching the device, and its
host-side RoPE table matches the CPU oracle's restatement of rope.h."""
import ctypes
import os
import re

import numpy as np
import pytest

import qib200 as Q
import qi_oracle as O


def declared_functions():
    src = open(Q.HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(qi_[a-z0-9_]+)\s*\(", src)))


def test_library_loads_and_exports_all_symbols():
    L = Q.lib()
    names = declared_functions()
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_status_strings():
    L = Q.lib()
    assert L.qi_status_string(0) == b"ok"
    for st in range(1, 9):
        assert L.qi_status_string(st) not in (b"ok", b"unknown status")
    assert L.qi_status_string(99) == b"unknown status"


def test_argument_validation_without_device():
    L = Q.lib()
    null = ctypes.c_void_p(0)
    assert L.qi_quantize_weight(null, 4, 64, null, null, null) == 1
    assert L.qi_fwht_quantize(null, 4, 64, 64, null, null, null) == 1
    assert L.qi_linear_i8(null, null, 4, 64, null, null, 32, null, 0, null, null, 32, null) == 1
    assert L.qi_linear_i8(null, null, 4, 64, null, null, 32, null, 7, null, null, 32, null) == 1
    assert L.qi_sage_attention(null, null, null, null, 0.1, 1, 8, 64, null) == 5  # head_dim 64 unsupported
    p16 = ctypes.c_void_p(256)
    assert L.qi_sage_attention(p16, p16, p16, p16, 0.1, 1, 131073, 128, null) == 5  # longer than the kernel takes
    assert L.qi_forward(null, null, 1, null, 0.0, null, 8, null, 8, 8, null, null) == 1
    assert L.qi_model_create(null, 1, null, null, None) == 1
    assert L.qi_rope_table(8, 8, 8, null) == 1
    # the allocation-free linear checks its arguments and its scratch limits
    # (4096 rows, 4 Mi codes) before it looks for a device; pointers that are
    # never dereferenced stand in for buffers
    p = ctypes.c_void_p(256)
    assert L.qi_linear_i8_f32in_noalloc(null, 4, 256, null, null, 64, null, 0, null, null) == 1
    assert L.qi_linear_i8_f32in_noalloc(p, 4097, 256, p, p, 64, null, 0, p, null) == 5
    assert L.qi_linear_i8_f32in_noalloc(p, 4096, 2048, p, p, 64, null, 0, p, null) == 5
    assert L.qi_linear_i8_f32in_noalloc(p, 0, 256, p, p, 64, null, 0, p, null) == 0
    # shapes and alignments the quantizer or GEMM would reject are refused
    # before anything is launched or the shared scratch is touched
    odd = ctypes.c_void_p(264)  # 8-byte aligned only
    assert L.qi_linear_i8_f32in_noalloc(p, 4, 100, p, p, 64, null, 0, p, null) == 1  # K % 16
    assert L.qi_linear_i8_f32in_noalloc(p, 4, 256, p, p, 48, null, 0, p, null) == 1  # N % 32 (GEMM path)
    assert L.qi_linear_i8_f32in_noalloc(p, 4, 256, odd, p, 64, null, 0, p, null) == 2  # w alignment
    assert L.qi_linear_i8_f32in_noalloc(p, 4, 256, p, odd, 64, null, 0, p, null) == 2  # w_scales alignment
    assert L.qi_linear_i8_f32in_noalloc(p, 4, 256, p, p, 64, null, 0, odd, null) == 2  # out alignment
    assert L.qi_linear_i8_f32in_noalloc(p, 1, 16384, p, p, 64, null, 0, p, null) == 5  # K beyond the quantizer


def test_null_handles_and_buffers_are_rejected_without_device():
    """Every entry point checks its handles and buffers before any CUDA call:
    null ones give QI_ERR_ARG (1); destroying a null handle is a no-op; the
    read-only queries answer 0 for a null handle."""
    L = Q.lib()
    null = None
    assert L.qi_version() > 0
    assert L.qi_ctx_create(0, null) == 1
    assert L.qi_ctx_destroy(null) == 0
    assert L.qi_ctx_check(null) == 1
    assert L.qi_ctx_last_launch_count(null) == 0
    assert L.qi_ctx_set_profiling(null, 1) == 1
    assert L.qi_ctx_profile(null, null, null, 0) == 1
    assert L.qi_selftest_wait_timeout(null, 1000, null) == 1
    assert L.qi_comm_unique_id(null) == 1
    assert L.qi_ctx_set_comm(null, null, 0, 1) == 1
    assert L.qi_model_load_safetensors(null, null, null) == 1
    assert L.qi_model_num_blocks(null) == 0
    assert L.qi_model_destroy(null) == 0
    assert L.qi_forward_blocks(null, null, 2, 16, 8, null, null, 500.0, null, 0, 1, null) == 1
    assert L.qi_layer_norm_modulate(null, null, null, null, 4, 64, 1e-6, null) == 1
    assert L.qi_rms_norm(null, null, null, 4, 64, 1e-6, null) == 1
    assert L.qi_sage_quantize(null, null, 1, 64, null, null, null, null, null, null) == 1
    assert L.qi_cfg_euler_step(null, null, null, 4.0, 0.5, 0.4, 8, 8, null, null) == 1
    assert L.qi_layer_norm_modulate_quantize(null, null, null, 4, 3072, 1e-6, null, null, null) == 1
    assert L.qi_qk_norm_rope(null, null, null, null, 1, 16, 8, null, null) == 1
    assert L.qi_qkv_norm_rope_i8(*([null] * 12), 1, 16, 8, null, null) == 1
    assert L.qi_ctx_set_fused_qkv_epilogue(null, 1) == 1
    assert L.qi_alloc_count() >= 0


@pytest.mark.parametrize("h,w,n_txt", [(8, 8, 8), (128, 128, 256), (166, 166, 256), (7, 9, 5)])
def test_rope_table_matches_oracle(h, w, n_txt):
    a = Q.rope_table(h, w, n_txt)
    b = O.rope_table(h, w, n_txt)
    assert a.shape == b.shape == (n_txt + ((h + 1) // 2) * ((w + 1) // 2), 64, 2, 2)
    np.testing.assert_array_equal(a, b)


def test_rope_table_matches_reference_digest(golden_dir):
    import hashlib
    path = os.path.join(golden_dir, "rope.npz")
    if not os.path.exists(path):
        pytest.skip("golden fixtures not generated")
    g = np.load(path)
    for key in g.files:
        if not key.startswith("sha256_"):
            continue
        h, w, n = (int(v) for v in key.split("_")[1:])
        assert hashlib.sha256(Q.rope_table(h, w, n).tobytes()).digest() == bytes(g[key]), key
