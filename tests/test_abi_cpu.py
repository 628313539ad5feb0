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


def test_argmax_validation():
    """Argmax.swift:24-37: axis must be the last one, indices int32 with one
    element per row; short rows route to `argmax`, long ones to `argmax_row`."""
    K, E, D = pc.Kernels, pc.PopcornError, pc.DataType
    k = K.Argmax(fake([2, 31], D.f32), fake([2], D.i32))
    assert k.function_names == ["argmax"]
    assert K.Argmax(fake([2, 32], D.bf16), fake([2], D.i32)).function_names == ["argmax_row"]
    expect_error(E.tensorInvalidAxis, K.Argmax, fake([2, 3], D.f32), fake([3], D.i32), axis=0)
    expect_error(E.tensorShapeMismatch, K.Argmax, fake([2, 3], D.f32), fake([3], D.i32))
    expect_error(E.unsupportedDataTypeCombination, K.Argmax, fake([2, 3], D.f32), fake([2], D.f32))


def test_rope_validation():
    """RopeBuildCosSin.swift:31-50 and RopeApply.swift:19-64."""
    K, E, D = pc.Kernels, pc.PopcornError, pc.DataType
    t = fake([5, 8], D.f32)
    K.RopeBuildCosSin(fake([5], D.i32), fake([8], D.f32), t, t)
    expect_error(E.tensorShapeMismatch, K.RopeBuildCosSin, fake([5], D.i32), fake([8], D.f32), t,
                 fake([5, 7], D.f32))
    expect_error(E.tensorInvalidRank, K.RopeBuildCosSin, fake([5], D.i32), fake([8], D.f32), fake([40], D.f32),
                 fake([40], D.f32))
    expect_error(E.tensorShapeMismatch, K.RopeBuildCosSin, fake([4], D.i32), fake([8], D.f32), t, t)
    expect_error(E.tensorShapeMismatch, K.RopeBuildCosSin, fake([5], D.i32), fake([7], D.f32), t, t)
    x = fake([1, 5, 2, 16], D.bf16)
    assert K.RopeApply(x, t, t, x).function_names == ["rope_apply_f32_tables_bf16"]
    tb = fake([5, 8], D.bf16)
    assert K.RopeApply(x, tb, tb, x).function_names == ["rope_apply_bf16"]
    expect_error(E.unsupportedDataTypeCombination, K.RopeApply, fake([1, 5, 2, 16], D.f32), tb, tb,
                 fake([1, 5, 2, 16], D.f32))
    expect_error(E.tensorShapeMismatch, K.RopeApply, fake([1, 5, 2, 15], D.f32), fake([5, 7], D.f32),
                 fake([5, 7], D.f32), fake([1, 5, 2, 15], D.f32))
    expect_error(E.tensorShapeMismatch, K.RopeApply, x, fake([4, 8], D.f32), fake([4, 8], D.f32), x)
    expect_error(E.tensorInvalidRank, K.RopeApply, fake([5, 2, 16], D.bf16), t, t, fake([5, 2, 16], D.bf16))
    # the fused per-head norm + RoPE of a decode step
    q = fake([1, 4, 1, 16], D.bf16)
    kc = fake([1, 2, 32, 16], D.bf16)
    w = fake([16], D.f32)
    tq = fake([32, 8], D.f32)  # a row per position
    k = K.QKNormRope(q, kc, kc, w, w, tq, tq, offset=31)
    acc = [b[3] for b in k.tensors][:3]
    assert acc == [pc.Access.readWrite] * 3
    K.QKNormRope(q, kc, kc, w, w, fake([1, 8], D.f32), fake([1, 8], D.f32), offset=31)  # the step's row
    expect_error(E.tensorShapeMismatch, K.QKNormRope, q, kc, kc, w, w, tq, tq, offset=32)
    expect_error(E.tensorShapeMismatch, K.QKNormRope, q, kc, kc, w, w, t, t, offset=5)  # beyond the table
    expect_error(E.unsupportedDataTypeCombination, K.QKNormRope, q, kc, kc, fake([16], D.bf16), w, tq, tq)


def test_scalar_mul_validation():
    K, E, D = pc.Kernels, pc.PopcornError, pc.DataType
    assert K.ScalarMul(fake([4], D.f16), by=2.0, into=fake([4], D.f16)).function_names == ["scalar_mul_f16"]
    expect_error(E.tensorShapeMismatch, K.ScalarMul, fake([4], D.f32), by=2.0, into=fake([5], D.f32))
    expect_error(E.unsupportedDataTypeCombination, K.ScalarMul, fake([4], D.i32), by=2.0, into=fake([4], D.i32))


def _aq(n, k, sdt=pc.DataType.bf16, bias=True, bits=4, group=64, packed_dt=pc.DataType.u32):
    return pc.AffineQuantizedTensor(fake([n, k // 8], packed_dt), fake([n, k // 64], sdt),
                                    fake([n, k // 64], sdt) if bias else None, (n, k), bits=bits,
                                    group_size=group)


def test_affine_quantized_matmul_validation():
    """Matmul.swift:99-131, 279-351 and AffineQuantizedTensor.swift:22-50."""
    K, E, D = pc.Kernels, pc.PopcornError, pc.DataType
    x = fake([1, 256], D.bf16)
    k = K.Matmul(x, _aq(32, 256), fake([1, 32], D.bf16))
    assert k.function_names == ["aq_qmv_fast_bf16_bf16_bf16_b4_g64"]
    assert K.Matmul(fake([3, 256], D.f32), _aq(32, 256), fake([3, 32], D.f32)).function_names == \
        ["aq_matvec_simd4_f32_bf16_f32_b4_g64"]
    K.Matmul(x, _aq(32, 256, bias=False), fake([1, 32], D.f32))
    expect_error(E.tensorShapeMismatch, K.Matmul, fake([1, 192], D.bf16), _aq(32, 256), fake([1, 32], D.bf16))
    expect_error(E.tensorShapeMismatch, K.Matmul, x, _aq(32, 256), fake([1, 31], D.bf16))
    expect_error(E.unsupportedDataTypeCombination, K.Matmul, x, _aq(32, 256, bits=8), fake([1, 32], D.bf16))
    expect_error(E.unsupportedDataTypeCombination, K.Matmul, x, _aq(32, 256, group=32), fake([1, 32], D.bf16))
    expect_error(E.unsupportedDataTypeCombination, K.Matmul, x, _aq(32, 256, packed_dt=D.i32),
                 fake([1, 32], D.bf16))
    expect_error(E.unsupportedDataTypeCombination, K.Matmul, fake([1, 256], D.f16), _aq(32, 256),
                 fake([1, 32], D.f16))
    expect_error(E.tensorInvalidRank, K.Matmul, fake([256], D.bf16), _aq(32, 256), fake([1, 32], D.bf16))
    with pytest.raises(pc.PopcornError):  # scales and biases must agree
        pc.AffineQuantizedTensor(fake([32, 32], D.u32), fake([32, 4], D.bf16), fake([32, 4], D.f16), (32, 256))


def test_embedding_gather_validation():
    """EmbeddingGather.swift:12-95."""
    K, E, D = pc.Kernels, pc.PopcornError, pc.DataType
    ids = fake([3], D.i32)
    assert K.EmbeddingGather(ids, fake([10, 64], D.bf16), fake([3, 64], D.f32)).function_names == \
        ["embedding_gather_bf16_to_f32"]
    expect_error(E.unsupportedDataTypeCombination, K.EmbeddingGather, ids, fake([10, 64], D.f16),
                 fake([3, 64], D.f32))
    expect_error(E.tensorShapeMismatch, K.EmbeddingGather, ids, fake([10, 64], D.f32), fake([4, 64], D.f32))
    expect_error(E.tensorInvalidRank, K.EmbeddingGather, ids, fake([640], D.f32), fake([3, 64], D.f32))
    q = _aq(1000, 256)
    assert K.EmbeddingGather(ids, q, fake([3, 256], D.bf16)).function_names == \
        ["aq_embedding_gather_bf16_bf16_b4_g64"]
    expect_error(E.unsupportedDataTypeCombination, K.EmbeddingGather, fake([3], D.i64), q, fake([3, 256], D.bf16))
    expect_error(E.tensorShapeMismatch, K.EmbeddingGather, ids, q, fake([3, 255], D.bf16))
    expect_error(E.tensorInvalidRank, K.EmbeddingGather, fake([1, 3], D.i32), q, fake([3, 256], D.bf16))


def test_fused_affine_quantized_validation():
    K, E, D = pc.Kernels, pc.PopcornError, pc.DataType
    x = fake([1, 256], D.bf16)
    nw = fake([256], D.f32)
    expect_error(E.unsupportedDataTypeCombination, K.AqRMSNormMatmul, fake([1, 256], D.f32), nw, _aq(32, 256),
                 fake([1, 32], D.f32))
    expect_error(E.tensorShapeMismatch, K.AqMatmulResidual, x, _aq(32, 256), fake([1, 31], D.bf16),
                 fake([1, 32], D.bf16))
    expect_error(E.tensorShapeMismatch, K.AqGatedMLP, x, nw, _aq(40, 256), fake([1, 20], D.bf16))
    expect_error(E.unsupportedDataTypeCombination, K.AqRMSNormMatmul, x, fake([256], D.bf16), _aq(32, 256),
                 fake([1, 32], D.bf16))


def test_batched_helper_validation():
    K, E, D = pc.Kernels, pc.PopcornError, pc.DataType
    qkv = fake([4, (8 + 2 * 2) * 64], D.bf16)
    q = fake([4, 8, 1, 64], D.bf16)
    kc = fake([4, 2, 16, 64], D.bf16)
    k = K.QKVScatter(qkv, q, kc, kc, offset=15)
    assert [b[3] for b in k.tensors] == [pc.Access.read] + [pc.Access.write] * 3
    expect_error(E.tensorShapeMismatch, K.QKVScatter, qkv, q, kc, kc, offset=16)
    expect_error(E.tensorShapeMismatch, K.QKVScatter, fake([4, 700], D.bf16), q, kc, kc)
    expect_error(E.unsupportedDataTypeCombination, K.QKVScatter, qkv, fake([4, 8, 1, 64], D.f16), kc, kc)
    K.GatedActivation(fake([3, 64], D.f16), fake([3, 32], D.f16), activation=1)
    expect_error(E.tensorShapeMismatch, K.GatedActivation, fake([3, 64], D.f16), fake([3, 31], D.f16))
    expect_error(E.unsupportedDataTypeCombination, K.GatedActivation, fake([3, 64], D.f16), fake([3, 32], D.f16),
                 activation=7)
    a = fake([2, 128], D.bf16)
    K.AddRMSNorm(a, a, fake([128], D.f32), a, a)
    expect_error(E.tensorShapeMismatch, K.AddRMSNorm, a, fake([2, 127], D.bf16), None, a, a)
    expect_error(E.unsupportedDataTypeCombination, K.AddRMSNorm, a, a, fake([128], D.bf16), a, a)


def test_attention_mask_build_validation():
    K, E, D = pc.Kernels, pc.PopcornError, pc.DataType
    assert K.AttentionMaskBuild(fake([3, 5], D.f32)).function_names == ["attention_mask_build"]
    expect_error(E.tensorInvalidRank, K.AttentionMaskBuild, fake([15], D.f32))
    expect_error(E.unsupportedDataTypeCombination, K.AttentionMaskBuild, fake([3, 5], D.f16))
