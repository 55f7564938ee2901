"""CPU tests of the C ABI: libinf.so loads, exports every function include/inf.h declares,
and the host-only parts (presets, arenas, byte model, error strings) behave without a GPU."""
import ctypes as C
import os
import re

import pytest

import infb200 as I

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    src = open(os.path.join(ROOT, "include", "inf.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    names = re.findall(r"^\s*(?:const\s+)?[A-Za-z_][A-Za-z0-9_]*\**\s+\**([a-z_][a-z0-9_]*)\s*\(", src, flags=re.M)
    return sorted(set(names))


def test_header_declares_the_binding_surface():
    decl = declared_functions()
    assert "inf_model_build" in decl and "inf_generate" in decl and "exec_ctx_create" in decl
    assert set(decl) == set(I.EXPORTS), set(decl) ^ set(I.EXPORTS)


def test_library_exports_every_declared_symbol():
    L = I.lib()
    for name in declared_functions():
        assert hasattr(L, name), name


def test_presets():
    c3 = I.preset(3)
    assert (c3.vocab_size, c3.dim, c3.n_layers, c3.n_heads, c3.n_kv_heads, c3.head_dim, c3.ffn_dim) == \
        (128256, 4096, 32, 32, 8, 128, 14336)
    assert c3.dtype == I.BF16 and abs(c3.rope_theta - 5e5) < 1 and c3.max_seq >= 2048 + 1024
    c1 = I.preset(1)
    assert (c1.dim, c1.n_layers, c1.head_dim, c1.ffn_dim, c1.dtype) == (288, 6, 48, 768, I.F32)
    assert I.preset(4).max_batch == 64 and I.preset(5).max_seq >= 32768 + 128
    c6 = I.preset(6)  # the Gemma-4-E2B shape of the reference's src/model.cuh:9-14
    assert (c6.arch, c6.dim, c6.ffn_dim, c6.head_dim, c6.n_heads, c6.vocab_size, c6.n_layers, c6.ple_dim) == \
        (I.ARCH_GEMMA, 1536, 6144, 512, 8, 262144, 35, 256)
    with pytest.raises(I.InfError) as e:
        I.preset(9)
    assert e.value.code == 4


def test_gemma_config_rules_without_a_device():
    """Gemma-style models are bf16 and single-GPU; ple_dim and the soft-cap belong to them only."""
    L = I.lib()
    ctx, m = C.POINTER(I.ExecCtx)(), I.Model()
    for bad in (dict(dtype=I.F32), dict(tp_size=2), dict(ple_dim=12), dict(head_dim=1024)):
        c = I.preset(6, n_layers=1, vocab_size=1024, **bad)
        assert L.inf_model_build(C.byref(ctx), C.byref(m), C.byref(c), None, 0) in (9, 15), bad
    c = I.preset(3, n_layers=1, ple_dim=16)
    assert L.inf_model_build(C.byref(ctx), C.byref(m), C.byref(c), None, 0) == 9


def test_decode_bytes_model():
    c = I.preset(3)
    w = 32 * ((32 + 16) * 128 * 4096 + 4096 * 4096 + 3 * 14336 * 4096 + 2 * 4096) * 2 + 128256 * 4096 * 2 + 2 * 4096 * 2
    kv = 2 * 32 * 8 * 128 * 2 * (2560 + 1)
    assert I.decode_bytes(c, 2560) == w + kv
    assert abs(w / 1e9 - 15.01) < 0.01  # 15.01 GB of weights per token


def test_error_strings():
    L = I.lib()
    assert L.inf_error_string(0) == b"Success"
    assert L.inf_error_string(10) == b"ErrorTokenOutOfRange"
    assert L.inf_error_string(7) == b"ErrorGeneric"


def test_host_arena_semantics():
    L = I.lib()
    a = C.POINTER(I.HostArena)()
    assert L.arena_host_create(C.byref(a), 1 << 24, 1 << 16) == 0
    p0 = L.mem_arena_host_pos_get(a)
    ptr = C.c_void_p()
    assert L.arena_host_push(a, 100, C.byref(ptr)) == 0
    assert ptr.value % 8 == 0
    C.memset(ptr, 7, 100)
    big = C.c_void_p()
    assert L.arena_host_push(a, 1 << 20, C.byref(big)) == 0  # grows past the first commit
    C.memset(big, 1, 1 << 20)
    assert L.arena_host_push(a, 1 << 30, C.byref(big)) == 2  # ErrorArenaOutOfMemory
    L.arena_host_pop_at(a, p0)
    assert L.mem_arena_host_pos_get(a) == p0
    L.arena_host_pop(a, 1 << 40)  # never pops the header
    assert L.mem_arena_host_pos_get(a) >= 32
    assert L.arena_host_destroy(a) == 0


def test_exec_ctx_lifecycle_without_device():
    L = I.lib()
    ctx = C.POINTER(I.ExecCtx)()
    assert L.exec_ctx_create(C.byref(ctx)) == 0
    assert ctx.contents.dev_arena._d_ptr is None
    assert L.exec_ctx_create(C.byref(ctx)) == 3  # ErrorAlreadyInitialized
    assert L.exec_ctx_destroy(C.byref(ctx)) == 0
    assert not ctx
    assert L.exec_ctx_destroy(C.byref(ctx)) == 4  # ErrorInvalidValue


def test_model_build_rejects_bad_config_without_touching_the_device():
    c = I.preset(3)
    c.n_kv_heads = 5  # 32 % 5 != 0
    with pytest.raises(I.InfError) as e:
        I.Engine(c)
    assert e.value.code == 9  # ErrorBadConfig


def test_library_id_generator_matches_oracle():
    import oracle as O
    import numpy as np
    np.testing.assert_array_equal(I.synth_ids(1, 300, 128256), O.gen_ids(1, 300, 128256))
    lens = I.synth_uniform(2, I.STREAM_CTX_LEN, 64, 512, 4096)
    want = [O.uniform_u32(2, O.STREAM_CTX_LEN, i, 512, 4096) for i in range(64)]
    np.testing.assert_array_equal(lens, np.array(want, np.uint32))


def test_new_entry_points_reject_null_arguments_without_a_device():
    """Checkpoint, tokenizer, server and sampling entry points fail with ErrorInvalidValue (4) on
    missing arguments before touching anything."""
    L = I.lib()
    c = I.preset(1)
    n = I.u64()
    assert L.inf_safetensors_check(None, C.byref(c)) == 4
    assert L.inf_safetensors_check(b"x", None) == 4
    assert L.inf_config_from_json(None, C.byref(c)) == 4
    assert L.inf_tokenizer_build(None, None) == 4
    assert L.inf_tokenizer_destroy(None) == 4
    assert L.inf_tokenizer_encode(None, b"a", None, 0, C.byref(n)) == 4
    assert L.inf_tokenizer_decode(None, None, 0, None, 0, C.byref(n)) == 4
    assert L.inf_tokenizer_vocab_size(None) == 0
    assert L.inf_server_create(None, 0, C.byref(I.vp())) == 4
    assert L.inf_server_create_synthetic(0, 16, 10, 0, 0, C.byref(I.vp())) == 4
    assert L.inf_server_step(None, None) == 4
    assert L.inf_server_destroy(None) == 4
    assert L.inf_server_stats(None, None, None, None, None) == 4
    assert L.inf_set_sampling(None, None) == 4
    s = I.InfSampling(temperature=1.0, top_p=1.0)
    assert L.inf_set_sampling(C.byref(I.Model()), C.byref(s)) == 4  # no engine


def test_memory_wrappers_keep_the_reference_return_conventions_without_a_device():
    """src/cuda/api/cuda_mem_wrapper.cuh:10-16: the b32 wrappers answer 1 for success and 0 for
    failure, cu_memcpy_htd / cu_memcpy_dth return Error_t.  Without a GPU every pointer is rejected
    (or the CUDA call fails) and each wrapper says so without aborting."""
    L = I.lib()
    buf = (C.c_uint8 * 64)()
    p = I.vp(1234)
    assert L.cu_malloc(None, 16) == 0
    assert L.cu_malloc(C.byref(p), 16) == 0 and not p.value  # no device to allocate on
    assert L.cu_free(buf) == 0
    assert L.cu_memset(buf, 0, 64) == 0
    assert L.cu_memcpy_htd_async(buf, buf, 64, None) == 0
    assert L.cu_memcpy_htd(buf, buf, 64) == 6   # ErrorInvalidDevPtr: dst is host memory
    assert L.cu_memcpy_dth(buf, buf, 64) == 5   # ErrorInvalidHostPtr, as the reference answers
    assert L.cu_host_register_read_only(None, 64) == 0
    assert b"cu_host_register_read_only" in I.lib().inf_last_error_detail()
