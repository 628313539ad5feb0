"""C-ABI tests that need no GPU: the library loads, exports every symbol the
header declares, and its host-side validation returns the reference's error
codes before anything touches a device."""
import ctypes
import re

import numpy as np
import pytest

from popcorn_b200 import _native as N
import popcorn_b200 as pc

FAKE = 0x7F0000000000  # never dereferenced: validation fails or no launch happens


def fake(shape, dtype, ptr=FAKE):
    return pc.Tensor(ptr, shape, dtype)


def test_library_loads_and_exports_header_symbols():
    L = N.lib()
    syms = N.header_symbols()
    assert len(syms) >= 45
    for s in syms:
        assert hasattr(L, s), s


def test_exports_only_the_c_abi():
    import subprocess
    out = subprocess.run(["nm", "-D", "--defined-only", N.LIB_PATH], capture_output=True, text=True).stdout
    exported = sorted({ln.split()[-1] for ln in out.splitlines() if " T " in ln})
    assert exported == N.header_symbols()


def test_dtype_strides_match_reference():
    # Tensor.DataType.stride, Tensor.swift:152-159
    exp = {pc.DataType.u8: 1, pc.DataType.i8: 1, pc.DataType.u16: 2, pc.DataType.i16: 2, pc.DataType.f16: 2,
           pc.DataType.bf16: 2, pc.DataType.u32: 4, pc.DataType.i32: 4, pc.DataType.f32: 4, pc.DataType.u64: 8,
           pc.DataType.i64: 8}
    for dt, s in exp.items():
        assert dt.stride == s
    assert N.lib().pc_dtype_stride(99) == 0


def test_scratch_spec_byte_count():
    # Internals/KernelResourceTests.swift:5-9
    assert pc.ScratchSpec([2, 3, 4], pc.DataType.f32).byte_count == 96
    assert pc.ScratchSpec([], pc.DataType.bf16).byte_count == 2
    assert pc.ScratchSpec([0, 5], pc.DataType.f32).byte_count == 1


def test_route_matches_reference():
    # FlashAttention.route, FlashAttention.swift:109-113
    FA = pc.Kernels.FlashAttention
    assert FA.route(1, 256) == FA.DECODING
    assert FA.route(2, 256) == FA.PLAIN
    assert FA.route(31, 256) == FA.PLAIN
    assert FA.route(32, 256) == FA.TENSOR
    assert FA.route(32, 256, pc.DataType.f32) == FA.PLAIN


def expect_error(code, fn, *a, **kw):
    with pytest.raises(pc.PopcornError) as e:
        fn(*a, **kw)
    assert e.value.code == code, e.value.message
    assert e.value.message
    return e.value


def test_flash_attention_validation():
    K = pc.Kernels
    q = fake([1, 8, 1, 256], pc.DataType.f16)
    kv = fake([1, 4, 64, 256], pc.DataType.f16)
    out = fake([1, 8, 1, 256], pc.DataType.f16)
    k = K.FlashAttention(q, kv, kv, into=out, scale=1 / 16)
    assert k.name == "FlashAttention"
    assert k.function_names == ["flash_decoding_partial_f16", "flash_decoding_reduce_f16"]
    acc = [t[3] for t in k.tensors]
    assert acc == [pc.Access.read, pc.Access.read, pc.Access.read, pc.Access.write]
    # FlashAttention.swift:27-36, 59-83
    E = pc.PopcornError
    expect_error(E.tensorShapeMismatch, K.FlashAttention, fake([1, 6, 1, 256], pc.DataType.f16), kv, kv,
                 into=fake([1, 6, 1, 256], pc.DataType.f16), scale=1.0)
    expect_error(E.tensorShapeMismatch, K.FlashAttention, fake([1, 8, 1, 600], pc.DataType.f16),
                 fake([1, 4, 64, 600], pc.DataType.f16), fake([1, 4, 64, 600], pc.DataType.f16),
                 into=fake([1, 8, 1, 600], pc.DataType.f16), scale=1.0)
    expect_error(E.tensorInvalidRank, K.FlashAttention, fake([8, 1, 256], pc.DataType.f16), kv, kv, into=out,
                 scale=1.0)
    expect_error(E.tensorShapeMismatch, K.FlashAttention, q, kv, fake([1, 4, 63, 256], pc.DataType.f16), into=out,
                 scale=1.0)
    expect_error(E.tensorShapeMismatch, K.FlashAttention, q, kv, kv, into=fake([1, 8, 2, 256], pc.DataType.f16),
                 scale=1.0)
    expect_error(E.unsupportedDataTypeCombination, K.FlashAttention, fake([1, 8, 1, 256], pc.DataType.i32), kv, kv,
                 into=out, scale=1.0)


def test_kv_cache_write_validation():
    K, E = pc.Kernels, pc.PopcornError
    src = fake([1, 1, 2, 2], pc.DataType.f32)
    cache = fake([1, 1, 4, 2], pc.DataType.f32)
    assert K.KVCacheWrite(src, cache, offset=2).function_names == ["kv_cache_write"]
    assert K.KVCacheWrite(fake([1, 1, 2, 2], pc.DataType.f32), fake([1, 1, 4, 2], pc.DataType.bf16),
                          offset=0).function_names == ["kv_cache_write_f32_to_bf16"]
    expect_error(E.tensorShapeMismatch, K.KVCacheWrite, src, cache, offset=3)
    expect_error(E.tensorShapeMismatch, K.KVCacheWrite, src, cache, offset=-1)
    expect_error(E.tensorShapeMismatch, K.KVCacheWrite, src, fake([1, 2, 4, 2], pc.DataType.f32), offset=0)
    expect_error(E.unsupportedDataTypeCombination, K.KVCacheWrite, fake([1, 1, 2, 2], pc.DataType.bf16),
                 fake([1, 1, 4, 2], pc.DataType.f32), offset=0)
    expect_error(E.tensorInvalidRank, K.KVCacheWrite, fake([2, 2], pc.DataType.f32), cache, offset=0)


def test_rmsnorm_validation():
    K, E = pc.Kernels, pc.PopcornError
    x = fake([3, 8], pc.DataType.bf16)
    w = fake([8], pc.DataType.f32)
    assert K.RMSNorm(x, w, into=fake([3, 8], pc.DataType.bf16), eps=1e-6).function_names == ["rmsnorm_bf16"]
    # RMSNorm.swift:47-64
    expect_error(E.tensorInvalidAxis, K.RMSNorm, x, w, into=fake([3, 8], pc.DataType.bf16), axis=0)
    expect_error(E.tensorShapeMismatch, K.RMSNorm, x, w, into=fake([3, 9], pc.DataType.bf16))
    expect_error(E.tensorShapeMismatch, K.RMSNorm, x, fake([7], pc.DataType.f32), into=fake([3, 8], pc.DataType.bf16))
    expect_error(E.unsupportedDataTypeCombination, K.RMSNorm, fake([3, 8], pc.DataType.i32), None,
                 into=fake([3, 8], pc.DataType.i32))
    # weight shape equal to x is accepted, as in the reference
    K.RMSNorm(x, fake([3, 8], pc.DataType.f32), into=fake([3, 8], pc.DataType.bf16))


def test_matmul_validation_and_routing():
    K, E = pc.Kernels, pc.PopcornError
    x = fake([1, 64], pc.DataType.bf16)
    w = fake([32, 64], pc.DataType.bf16)
    assert K.Matmul(x, w, into=fake([1, 32], pc.DataType.bf16), transpose_b=True).function_names == [
        "matvec_nk_bf16_bf16_bf16"]
    assert K.Matmul(fake([4, 64], pc.DataType.f32), fake([64, 32], pc.DataType.f32),
                    into=fake([4, 32], pc.DataType.f32)).function_names == ["matmul"]
    # Matmul.swift:69-91
    expect_error(E.tensorInvalidRank, K.Matmul, fake([64], pc.DataType.bf16), w, into=fake([1, 32], pc.DataType.bf16))
    expect_error(E.tensorShapeMismatch, K.Matmul, x, fake([32, 63], pc.DataType.bf16),
                 into=fake([1, 32], pc.DataType.bf16), transpose_b=True)
    expect_error(E.tensorShapeMismatch, K.Matmul, x, w, into=fake([1, 31], pc.DataType.bf16), transpose_b=True)
    expect_error(E.unsupportedDataTypeCombination, K.Matmul, fake([2, 64], pc.DataType.bf16),
                 fake([64, 32], pc.DataType.f32), into=fake([2, 32], pc.DataType.f32))


def test_elementwise_validation():
    K, E = pc.Kernels, pc.PopcornError
    a = fake([8], pc.DataType.f32)
    assert K.GeluTanh(a, into=fake([8], pc.DataType.f32)).function_names == ["gelu_tanh"]
    assert K.Add(fake([8], pc.DataType.bf16), fake([8], pc.DataType.bf16),
                 into=fake([8], pc.DataType.bf16)).function_names == ["add_bf16"]
    expect_error(E.tensorShapeMismatch, K.GeluTanh, a, into=fake([9], pc.DataType.f32))
    expect_error(E.tensorShapeMismatch, K.Mul, a, fake([4], pc.DataType.f32), into=a)
    expect_error(E.unsupportedDataTypeCombination, K.Add, a, fake([8], pc.DataType.f16), into=a)


def test_fused_validation():
    K, E = pc.Kernels, pc.PopcornError
    x = fake([1, 64], pc.DataType.bf16)
    w = fake([32, 64], pc.DataType.bf16)
    nw = fake([64], pc.DataType.f32)
    K.RMSNormMatmul(x, nw, w, into=fake([1, 32], pc.DataType.bf16))
    expect_error(E.unsupportedDataTypeCombination, K.RMSNormMatmul, x, fake([64], pc.DataType.bf16), w,
                 into=fake([1, 32], pc.DataType.bf16))
    expect_error(E.tensorShapeMismatch, K.GatedMLP, x, w, fake([32, 63], pc.DataType.bf16),
                 into=fake([1, 32], pc.DataType.bf16))
    q = fake([1, 2, 1, 16], pc.DataType.bf16)
    kc = fake([1, 1, 8, 16], pc.DataType.bf16)
    K.QKVProjection(x, nw, fake([64, 64], pc.DataType.bf16), q, kc, kc, offset=7)
    expect_error(E.tensorShapeMismatch, K.QKVProjection, x, nw, fake([64, 64], pc.DataType.bf16), q, kc, kc, offset=8)
    expect_error(E.tensorShapeMismatch, K.QKVProjection, x, nw, fake([60, 64], pc.DataType.bf16), q, kc, kc, offset=0)


def test_null_device_pointer_rejected():
    E = pc.PopcornError
    expect_error(E.tensorShapeMismatch, pc.Kernels.GeluTanh, pc.Tensor(0, [4], pc.DataType.f32),
                 into=fake([4], pc.DataType.f32))


def test_library_create_without_gpu_fails_cleanly():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(pc.PopcornError) as e:
        pc.KernelLibrary(0)
    assert -1019 <= e.value.code <= -1013


def test_error_message_is_thread_local():
    import threading
    msgs = {}

    def worker(name, shape):
        try:
            pc.Kernels.GeluTanh(fake([4], pc.DataType.f32), into=fake(shape, pc.DataType.f32))
        except pc.PopcornError as e:
            msgs[name] = e.message

    ts = [threading.Thread(target=worker, args=("a", [5])), threading.Thread(target=worker, args=("b", [6]))]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    assert "[5]" in msgs["a"] and "[6]" in msgs["b"]
