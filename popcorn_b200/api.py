"""Python mirror of Popcorn's public surface over the C ABI.

Same names, argument meaning and error behaviour as the reference's Swift
API (Sources/Popcorn/*.swift), so that callers and tests read like the
reference's own:

    library = KernelLibrary(device=0)
    encoder = KernelCommandEncoder(library, stream=torch.cuda.current_stream(),
                                   scratch=ScratchPool())
    encoder.encode(Kernels.FlashAttention(q, k, v, into=out, scale=1/16))

Kernel constructors validate eagerly and raise PopcornError with the
reference's codes (PopcornError.swift:23-42). Tensors wrap caller-owned
device memory (torch tensors here) at offset 0, as Tensor.swift:5-22 does.
Every computation runs in libpopcorn_cuda.so on the GPU.
"""
import ctypes
import enum

from . import _native as N


class PopcornError(Exception):
    """PopcornError (PopcornError.swift:6-76): a code and a message."""

    constantAllocationFailed = -1001
    tensorAllocationFailed = -1003
    kernelFunctionNotFound = -1006
    tensorShapeMismatch = -1007
    tensorInvalidRank = -1008
    tensorInvalidAxis = -1009
    unsupportedDataTypeCombination = -1010
    workspaceExhausted = -1012
    gpuOutOfMemory = -1013
    gpuTimeout = -1014
    gpuPageFault = -1015
    gpuInvalidResource = -1016
    gpuDeviceRemoved = -1017
    gpuAccessRevoked = -1018
    gpuInternal = -1019

    def __init__(self, code, message):
        super().__init__("[%d] %s" % (code, message))
        self.code = code
        self.message = message

    def __eq__(self, other):  # PopcornError.swift:68-70: equal by code
        return isinstance(other, PopcornError) and other.code == self.code

    def __hash__(self):
        return hash(self.code)


def _check(status):
    if status != 0:
        msg = N.lib().pc_last_error_message()
        raise PopcornError(status, msg.decode() if msg else "")


class DataType(enum.IntEnum):
    """Tensor.DataType (Tensor.swift:135-177), same raw order."""

    u8 = 0
    u16 = 1
    u32 = 2
    u64 = 3
    i8 = 4
    i16 = 5
    i32 = 6
    i64 = 7
    f32 = 8
    f16 = 9
    bf16 = 10

    @property
    def stride(self):
        return N.lib().pc_dtype_stride(int(self))


def _torch_dtype_map():
    import torch
    return {torch.float32: DataType.f32, torch.float16: DataType.f16, torch.bfloat16: DataType.bf16,
            torch.int32: DataType.i32, torch.int64: DataType.i64, torch.uint8: DataType.u8,
            torch.int8: DataType.i8, torch.int16: DataType.i16, torch.uint32: DataType.u32}


class Access(enum.IntFlag):
    """Tensor.Access (Tensor.swift:182-199)."""

    read = 1
    write = 2
    readWrite = 3


class Tensor:
    """Tensor {buffer, shape, dataType} over caller-owned device memory."""

    def __init__(self, data_ptr, shape, dtype, owner=None):
        self.data_ptr = int(data_ptr)
        self.shape = tuple(int(s) for s in shape)
        self.dtype = DataType(dtype)
        self._owner = owner  # keeps the backing storage alive

    @classmethod
    def from_torch(cls, t, shape=None):
        """Wraps a contiguous CUDA torch tensor (bf16/f16/f32/i32/...)."""
        if not t.is_contiguous():
            raise PopcornError(PopcornError.tensorShapeMismatch, "tensor must be contiguous")
        dt = _torch_dtype_map().get(t.dtype)
        if dt is None:
            raise PopcornError(PopcornError.unsupportedDataTypeCombination, "unsupported torch dtype %s" % t.dtype)
        return cls(t.data_ptr(), tuple(t.shape) if shape is None else shape, dt, owner=t)

    @property
    def element_count(self):
        n = 1
        for s in self.shape:
            n *= s
        return n

    def c(self):
        d = N.pc_tensor()
        d.data = self.data_ptr or None
        d.dtype = int(self.dtype)
        d.rank = len(self.shape)
        if d.rank > N.PC_MAX_RANK:
            raise PopcornError(PopcornError.tensorInvalidRank, "rank %d > 8" % d.rank)
        for i, s in enumerate(self.shape):
            d.shape[i] = s
        return d


def _tc(t):
    """Tensor | torch.Tensor | None -> pointer to pc_tensor (or None)."""
    if t is None:
        return None
    if not isinstance(t, Tensor):
        t = Tensor.from_torch(t)
    return ctypes.pointer(t.c())


class AttentionMask:
    """AttentionMask (AttentionMask.swift:17-41)."""

    def __init__(self, kind, window=-1):
        self.kind = kind
        self.window = window

    @classmethod
    def causal_sliding_window(cls, window):
        return cls(1, window)

    def c(self):
        return N.pc_attention_mask(self.kind, self.window)


AttentionMask.causal = AttentionMask(0)
AttentionMask.bidirectional = AttentionMask(2)


class ScratchSpec:
    """ScratchSpec (ScratchSpec.swift:10-26)."""

    def __init__(self, shape, dtype):
        self.shape = list(shape)
        self.dtype = DataType(dtype)

    @property
    def byte_count(self):
        arr = (ctypes.c_int64 * max(1, len(self.shape)))(*self.shape)
        return N.lib().pc_scratch_spec_byte_count(arr, len(self.shape), int(self.dtype))


class KernelLibrary:
    """KernelLibrary (KernelLibrary.swift:4-41)."""

    def __init__(self, device=0):
        h = ctypes.c_void_p()
        _check(N.lib().pc_library_create(int(device), ctypes.byref(h)))
        self._h = h
        self.device = int(device)

    def pipeline_state(self, function_name):
        """Returns the cached handle for a kernel function; -1006 if unknown."""
        out = ctypes.c_void_p()
        _check(N.lib().pc_library_lookup(self._h, function_name.encode(), ctypes.byref(out)))
        return out.value

    @property
    def function_names(self):
        L = N.lib()
        return [L.pc_library_function_name(self._h, i).decode() for i in range(L.pc_library_function_count(self._h))]

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and N._lib is not None:
            N.lib().pc_library_destroy(h)
            self._h = None


class KernelScratchAllocator:
    """KernelScratchAllocator protocol (KernelResources.swift:29-36).

    Subclasses implement borrow(length) -> (device_ptr, was_reused) and
    optionally release(ptr).
    """

    def borrow(self, length):
        raise NotImplementedError

    def release(self, ptr):
        pass

    def _c(self):
        def _borrow(ctx, length, out_ptr, out_reused):
            try:
                ptr, reused = self.borrow(int(length))
            except PopcornError as e:
                return e.code
            except Exception:
                return PopcornError.tensorAllocationFailed
            out_ptr[0] = ptr
            out_reused[0] = 1 if reused else 0
            return 0

        def _release(ctx, ptr):
            self.release(int(ptr) if ptr else 0)

        self._cb = (N.BORROW_FN(_borrow), N.RELEASE_FN(_release))
        return N.pc_scratch_allocator(None, self._cb[0], self._cb[1])


class ScratchPool(KernelScratchAllocator):
    """Best-fit reusing pool over torch device memory.

    Mirrors the runtime pool of the reference's example app
    (Examples/GemmaCLI/Sources/GemmaCLI/ScratchPool.swift:17-71): released
    buffers return to the pool and are lent again with was_reused = True.
    All work must be on one stream (stream order protects reuse).
    """

    def __init__(self, device=0):
        self.device = device
        self._free = []   # (size, tensor)
        self._live = {}   # ptr -> (size, tensor)
        self.borrows = 0
        self.reuses = 0

    def borrow(self, length):
        import torch
        self.borrows += 1
        best = None
        for i, (size, t) in enumerate(self._free):
            if size >= length and (best is None or size < self._free[best][0]):
                best = i
        if best is not None:
            size, t = self._free.pop(best)
            self._live[t.data_ptr()] = (size, t)
            self.reuses += 1
            return t.data_ptr(), True
        size = max(256, (length + 255) // 256 * 256)
        t = torch.empty(size, dtype=torch.uint8, device="cuda:%d" % self.device)
        self._live[t.data_ptr()] = (size, t)
        return t.data_ptr(), False

    def release(self, ptr):
        item = self._live.pop(ptr, None)
        if item is not None:
            self._free.append(item)


class FixedScratch(KernelScratchAllocator):
    """Hands out slices of one preallocated buffer (no allocation after setup).

    Every borrow in one encode gets a distinct slice; the cursor resets when
    all borrowed slices are released. Suitable under CUDA graph capture.
    """

    def __init__(self, nbytes, device=0):
        import torch
        self.buf = torch.empty(nbytes, dtype=torch.uint8, device="cuda:%d" % device)
        self.base = self.buf.data_ptr()
        self.size = nbytes
        self.cursor = 0
        self.live = 0

    def borrow(self, length):
        start = (self.cursor + 255) // 256 * 256
        if start + length > self.size:
            raise PopcornError(PopcornError.workspaceExhausted, "fixed scratch exhausted")
        self.cursor = start + length
        self.live += 1
        return self.base + start, True

    def release(self, ptr):
        self.live -= 1
        if self.live == 0:
            self.cursor = 0


class KernelCommandEncoder:
    """KernelCommandEncoder (KernelCommandEncoder.swift:5-168) on a CUDA stream."""

    def __init__(self, library, stream=None, scratch=None):
        self.library = library
        if stream is None:
            import torch
            stream = torch.cuda.current_stream(library.device)
        self.stream = stream
        sptr = stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream or 0)
        self.scratch = scratch
        sc = ctypes.pointer(scratch._c()) if scratch is not None else None
        h = ctypes.c_void_p()
        _check(N.lib().pc_encoder_create(library._h, ctypes.c_void_p(sptr), sc, ctypes.byref(h)))
        self._h = h
        self._hook = None

    def encode(self, *kernels):
        """encode(_:) / the KernelBuilder form: encodes each kernel in order."""
        for k in kernels:
            if isinstance(k, (list, tuple)):
                self.encode(*k)
            elif k is not None:
                _check(N.lib().pc_encoder_encode(self._h, k._h))

    def barrier(self):
        _check(N.lib().pc_encoder_barrier(self._h))

    @property
    def barrier_count(self):
        return N.lib().pc_encoder_barrier_count(self._h)

    @property
    def dispatch_count(self):
        return N.lib().pc_encoder_dispatch_count(self._h)

    def set_dispatch_hook(self, fn):
        """fn(function_name, phase, stream_ptr); phase 0 = will, 1 = did dispatch."""
        if fn is None:
            self._hook = None
            _check(N.lib().pc_encoder_set_dispatch_hook(self._h, N.HOOK_FN(), None))
            return
        self._hook = N.HOOK_FN(lambda ctx, name, phase, stream: fn(name.decode(), phase, stream))
        _check(N.lib().pc_encoder_set_dispatch_hook(self._h, self._hook, None))

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and N._lib is not None:
            N.lib().pc_encoder_destroy(h)
            self._h = None


class Kernel:
    """A validated kernel value (Kernel.swift:15-70)."""

    def __init__(self, creator, *args, keep=()):
        h = ctypes.c_void_p()
        _check(creator(*args, ctypes.byref(h)))
        self._h = h
        self._keep = keep

    @property
    def name(self):
        return N.lib().pc_kernel_name(self._h).decode()

    @property
    def function_names(self):
        return N.lib().pc_kernel_function_names(self._h).decode().split(";")

    @property
    def tensors(self):
        L = N.lib()
        out = []
        for i in range(L.pc_kernel_binding_count(self._h)):
            t = N.pc_tensor()
            acc = ctypes.c_int()
            _check(L.pc_kernel_binding(self._h, i, ctypes.byref(t), ctypes.byref(acc)))
            out.append((t.data or 0, tuple(t.shape[:t.rank]), DataType(t.dtype), Access(acc.value)))
        return out

    def set_l2_prefetch(self, slot, region, nbytes=None):
        """L2 prefetch hint: after issuing its own loads the kernel pulls
        `region` (a torch tensor or a device address, `nbytes` long) into L2."""
        if region is None:
            ptr, n = None, 0
        elif isinstance(region, int):
            ptr, n = region, int(nbytes)
        else:
            ptr = region.data_ptr()
            n = region.numel() * region.element_size() if nbytes is None else int(nbytes)
            self._keep = self._keep + (region,)
        _check(N.lib().pc_kernel_set_l2_prefetch(self._h, int(slot), ptr, n))
        return self

    HINT_KV_EARLY = 2

    def set_hint(self, hint, value=1):
        """Scheduling hint (pc_kernel_set_hint). HINT_KV_EARLY: decode
        attention may copy the K/V rows older than each sequence's newest
        before it waits for the previous kernel (which must write no other
        rows, nor seq_lens). Results never change."""
        _check(N.lib().pc_kernel_set_hint(self._h, int(hint), int(value)))
        return self

    def encode(self, encoder):
        encoder.encode(self)

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and N._lib is not None:
            N.lib().pc_kernel_destroy(h)
            self._h = None


def _keep(*ts):
    return tuple(t for t in ts if t is not None)


class AffineQuantizedTensor:
    """AffineQuantizedTensor (Quantization/AffineQuantizedTensor.swift): a
    logical [out_features, in_features] weight stored as unsigned `bits`-bit
    values packed little-endian into u32 words (packed_values [out, in / 8]
    for 4 bits) with one scale / bias per `group_size` consecutive inner
    values (scales, biases [out, in / group_size]; biases may be None).
    w = q * scale + bias."""

    def __init__(self, packed_values, scales, biases, shape, bits=4, group_size=64):
        if biases is not None and (biases.dtype != scales.dtype or tuple(biases.shape) != tuple(scales.shape)):
            raise PopcornError(-1007, "AffineQuantizedTensor scales and biases must share a data type and shape.")
        if len(shape) < 2:
            raise PopcornError(-1008, "AffineQuantizedTensor shape must have rank >= 2.")
        import torch
        self.packed_tensor = packed_values if isinstance(packed_values, torch.Tensor) else None
        if isinstance(packed_values, torch.Tensor) and packed_values.dtype == torch.int32:
            # the same 32-bit words, typed as the format's u32 storage
            packed_values = Tensor(packed_values.data_ptr(), tuple(packed_values.shape), DataType.u32,
                                   owner=packed_values)
        self.packed_values, self.scales, self.biases = packed_values, scales, biases
        self.shape = tuple(int(d) for d in shape)
        self.bits, self.group_size = int(bits), int(group_size)

    def c(self):
        """pc_affine_quantized, plus the pc_tensor structs it points to."""
        parts = [_tc(self.packed_values), _tc(self.scales), _tc(self.biases)]
        st = N.pc_affine_quantized()
        st.packed = ctypes.cast(parts[0], ctypes.c_void_p)
        st.scales = ctypes.cast(parts[1], ctypes.c_void_p)
        st.biases = ctypes.cast(parts[2], ctypes.c_void_p) if parts[2] is not None else None
        st.out_features, st.in_features = self.out_features, self.in_features
        st.bits, st.group_size = self.bits, self.group_size
        return st, parts

    @property
    def out_features(self):
        return self.shape[-2]

    @property
    def in_features(self):
        return self.shape[-1]


class Kernels:
    """The op namespace (public extension Kernels { ... })."""

    class FlashAttention(Kernel):
        """Kernels.FlashAttention(q:k:v:into:scale:mask:) (FlashAttention.swift:51-90)."""

        PLAIN, TENSOR, DECODING = 0, 1, 2

        def __init__(self, q, k, v, into, scale, mask=AttentionMask.causal, dims=None):
            L = N.lib()
            if dims is None:
                super().__init__(L.pc_kernel_flash_attention, _tc(q), _tc(k), _tc(v), _tc(into),
                                 ctypes.c_float(scale), mask.c(), keep=_keep(q, k, v, into))
            else:
                b, nq, nkv, sq, sk, hd = dims
                super().__init__(L.pc_kernel_flash_attention_dims, _tc(q), _tc(k), _tc(v), _tc(into), b, nq,
                                 nkv, sq, sk, hd, ctypes.c_float(scale), mask.c(), keep=_keep(q, k, v, into))

        @staticmethod
        def route(sq, hd, dtype=DataType.bf16):
            return N.lib().pc_flash_attention_route(sq, hd, int(dtype))

    class FlashDecodingRagged(Kernel):
        """Extension: per-sequence lengths over a [B,Nkv,Smax,Hd] cache."""

        def __init__(self, q, k_cache, v_cache, seq_lens, into, scale, mask=AttentionMask.causal):
            super().__init__(N.lib().pc_kernel_flash_decoding_ragged, _tc(q), _tc(k_cache), _tc(v_cache),
                             _tc(seq_lens), _tc(into), ctypes.c_float(scale), mask.c(),
                             keep=_keep(q, k_cache, v_cache, seq_lens, into))

    class KVCacheWrite(Kernel):
        """Kernels.KVCacheWrite(source:cache:offset:) (KVCacheWrite.swift:38-49)."""

        def __init__(self, source, cache, offset, dims=None):
            L = N.lib()
            if dims is None:
                super().__init__(L.pc_kernel_kv_cache_write, _tc(source), _tc(cache), offset,
                                 keep=_keep(source, cache))
            else:
                b, nkv, snew, smax, hd = dims
                super().__init__(L.pc_kernel_kv_cache_write_dims, _tc(source), _tc(cache), b, nkv, snew, smax, hd,
                                 offset, keep=_keep(source, cache))

    class RMSNorm(Kernel):
        """Kernels.RMSNorm(_:weight:into:axis:eps:addOneToWeight:) (RMSNorm.swift:39-70)."""

        def __init__(self, x, weight=None, into=None, axis=-1, eps=1e-6, add_one_to_weight=False, dims=None):
            L = N.lib()
            if dims is None:
                super().__init__(L.pc_kernel_rmsnorm, _tc(x), _tc(weight), _tc(into), axis, ctypes.c_float(eps),
                                 int(add_one_to_weight), keep=_keep(x, weight, into))
            else:
                rows, h = dims
                super().__init__(L.pc_kernel_rmsnorm_dims, _tc(x), _tc(weight), _tc(into), rows, h,
                                 ctypes.c_float(eps), int(add_one_to_weight), keep=_keep(x, weight, into))

    class Matmul(Kernel):
        """Kernels.Matmul(_:_:into:transposeB:) (Matmul.swift:68-93); with an
        AffineQuantizedTensor b, Kernels.Matmul(_:_:into:) (Matmul.swift:
        99-131): c = a . dequant(b)^T."""

        def __init__(self, a, b, into, transpose_b=False, dims=None):
            L = N.lib()
            if isinstance(b, AffineQuantizedTensor):
                super().__init__(L.pc_kernel_matmul_affine_quantized, _tc(a), _tc(b.packed_values), _tc(b.scales),
                                 _tc(b.biases), b.out_features, b.in_features, b.bits, b.group_size, _tc(into),
                                 keep=_keep(a, b.packed_values, b.scales, b.biases, into))
            elif dims is None:
                super().__init__(L.pc_kernel_matmul, _tc(a), _tc(b), _tc(into), int(transpose_b),
                                 keep=_keep(a, b, into))
            else:
                m, k, n = dims
                super().__init__(L.pc_kernel_matmul_dims, _tc(a), _tc(b), _tc(into), m, k, n, int(transpose_b),
                                 keep=_keep(a, b, into))

    class AqRMSNormMatmul(Kernel):
        """Extension: Matmul(RMSNorm(x), w) with a 4-bit AffineQuantizedTensor w."""

        def __init__(self, x, norm_weight, w, into, eps=1e-6, add_one_to_weight=False):
            st, parts = w.c()
            super().__init__(N.lib().pc_kernel_aq_rmsnorm_matmul, _tc(x), _tc(norm_weight), ctypes.c_float(eps),
                             int(add_one_to_weight), ctypes.byref(st), _tc(into),
                             keep=_keep(x, norm_weight, w.packed_values, w.scales, w.biases, into) + (st, parts))

    class AqMatmulResidual(Kernel):
        """Extension: Add(Matmul(x, w), residual) with a 4-bit w."""

        def __init__(self, x, w, residual, into):
            st, parts = w.c()
            super().__init__(N.lib().pc_kernel_aq_matmul_residual, _tc(x), ctypes.byref(st), _tc(residual),
                             _tc(into),
                             keep=_keep(x, w.packed_values, w.scales, w.biases, residual, into) + (st, parts))

    class AqGatedMLP(Kernel):
        """Extension: act(g) * u of [g; u] = Matmul(RMSNorm(x), w_gate_up),
        w_gate_up's rows interleaved in blocks of 8 (gate, up)."""

        def __init__(self, x, norm_weight, w_gate_up, into, eps=1e-6, add_one_to_weight=False, activation=0):
            st, parts = w_gate_up.c()
            super().__init__(N.lib().pc_kernel_aq_gated_mlp, _tc(x), _tc(norm_weight), ctypes.c_float(eps),
                             int(add_one_to_weight), ctypes.byref(st), int(activation), _tc(into),
                             keep=_keep(x, norm_weight, w_gate_up.packed_values, w_gate_up.scales, w_gate_up.biases,
                                        into) + (st, parts))

    class AqQKVProjection(Kernel):
        """Extension: RMSNorm -> 4-bit Matmul [q; k; v] -> q and the new K/V
        rows into the caches at the position."""

        def __init__(self, x, norm_weight, w_qkv, q_out, k_cache, v_cache, offset=0, position=None, eps=1e-6,
                     add_one_to_weight=False):
            st, parts = w_qkv.c()
            super().__init__(N.lib().pc_kernel_aq_qkv_projection, _tc(x), _tc(norm_weight), ctypes.c_float(eps),
                             int(add_one_to_weight), ctypes.byref(st), _tc(q_out), _tc(k_cache), _tc(v_cache),
                             int(offset), _tc(position),
                             keep=_keep(x, norm_weight, w_qkv.packed_values, w_qkv.scales, w_qkv.biases, q_out,
                                        k_cache, v_cache, position) + (st, parts))

    class EmbeddingGather(Kernel):
        """Kernels.EmbeddingGather(ids:table:into:) (EmbeddingGather.swift):
        rows of a dense table, or of an AffineQuantizedTensor dequantised on
        the fly."""

        def __init__(self, ids, table, into):
            L = N.lib()
            if isinstance(table, AffineQuantizedTensor):
                super().__init__(L.pc_kernel_embedding_gather_affine_quantized, _tc(ids), _tc(table.packed_values),
                                 _tc(table.scales), _tc(table.biases), table.out_features, table.in_features,
                                 table.bits, table.group_size, _tc(into),
                                 keep=_keep(ids, table.packed_values, table.scales, table.biases, into))
            else:
                super().__init__(L.pc_kernel_embedding_gather, _tc(ids), _tc(table), _tc(into),
                                 keep=_keep(ids, table, into))

    class GeluTanh(Kernel):
        def __init__(self, x, into):
            super().__init__(N.lib().pc_kernel_gelu_tanh, _tc(x), _tc(into), keep=_keep(x, into))

    class AttentionMaskBuild(Kernel):
        """Kernels.AttentionMaskBuild(mask:slidingWindow:) (AttentionMaskBuild.swift)."""

        def __init__(self, mask, sliding_window=None):
            super().__init__(N.lib().pc_kernel_attention_mask_build, _tc(mask),
                             -1 if sliding_window is None else int(sliding_window), keep=_keep(mask))

    class ScalarMul(Kernel):
        """Kernels.ScalarMul(_:by:into:) (ScalarMul.swift)."""

        def __init__(self, x, by, into):
            super().__init__(N.lib().pc_kernel_scalar_mul, _tc(x), ctypes.c_float(by), _tc(into), keep=_keep(x, into))

    class SiLU(Kernel):
        def __init__(self, x, into):
            super().__init__(N.lib().pc_kernel_silu, _tc(x), _tc(into), keep=_keep(x, into))

    class Mul(Kernel):
        def __init__(self, a, b, into):
            super().__init__(N.lib().pc_kernel_mul, _tc(a), _tc(b), _tc(into), keep=_keep(a, b, into))

    class Add(Kernel):
        def __init__(self, a, b, into):
            super().__init__(N.lib().pc_kernel_add, _tc(a), _tc(b), _tc(into), keep=_keep(a, b, into))

    # ---- fused decode ops (extensions) ----

    class RMSNormMatmul(Kernel):
        def __init__(self, x, norm_weight, w, into, eps=1e-6, add_one_to_weight=False):
            super().__init__(N.lib().pc_kernel_rmsnorm_matmul, _tc(x), _tc(norm_weight), ctypes.c_float(eps),
                             int(add_one_to_weight), _tc(w), _tc(into), keep=_keep(x, norm_weight, w, into))

    class GatedMLP(Kernel):
        GELU_TANH, SILU = 0, 1

        def __init__(self, x, w_gate, w_up, into, norm_weight=None, eps=1e-6, add_one_to_weight=False,
                     activation=0):
            super().__init__(N.lib().pc_kernel_gated_mlp, _tc(x), _tc(norm_weight), ctypes.c_float(eps),
                             int(add_one_to_weight), _tc(w_gate), _tc(w_up), int(activation), _tc(into),
                             keep=_keep(x, norm_weight, w_gate, w_up, into))

    class MatmulResidual(Kernel):
        def __init__(self, a, w, residual, into):
            super().__init__(N.lib().pc_kernel_matmul_residual, _tc(a), _tc(w), _tc(residual), _tc(into),
                             keep=_keep(a, w, residual, into))

    class QKVProjection(Kernel):
        def __init__(self, x, norm_weight, w_qkv, q_out, k_cache, v_cache, offset=0, position=None, eps=1e-6,
                     add_one_to_weight=False):
            super().__init__(N.lib().pc_kernel_qkv_projection, _tc(x), _tc(norm_weight), ctypes.c_float(eps),
                             int(add_one_to_weight), _tc(w_qkv), _tc(q_out), _tc(k_cache), _tc(v_cache),
                             int(offset), _tc(position),
                             keep=_keep(x, norm_weight, w_qkv, q_out, k_cache, v_cache, position))


    class Argmax(Kernel):
        """Kernels.Argmax(_:indices:axis:) (Argmax.swift:24-37)."""

        def __init__(self, x, indices, axis=-1):
            super().__init__(N.lib().pc_kernel_argmax, _tc(x), _tc(indices), int(axis), keep=_keep(x, indices))

    class RopeBuildCosSin(Kernel):
        """Kernels.RopeBuildCosSin(positions:invFreq:cosOut:sinOut:attentionScaling:)
        (RopeBuildCosSin.swift:31-50)."""

        def __init__(self, positions, inv_freq, cos_out, sin_out, attention_scaling=1.0):
            super().__init__(N.lib().pc_kernel_rope_build_cos_sin, _tc(positions), _tc(inv_freq), _tc(cos_out),
                             _tc(sin_out), ctypes.c_float(attention_scaling),
                             keep=_keep(positions, inv_freq, cos_out, sin_out))

    class RopeApply(Kernel):
        """Kernels.RopeApply(_:cos:sin:into:) (RopeApply.swift:48-64)."""

        def __init__(self, x, cos, sin, into):
            super().__init__(N.lib().pc_kernel_rope_apply, _tc(x), _tc(cos), _tc(sin), _tc(into),
                             keep=_keep(x, cos, sin, into))

    class QKNormRope(Kernel):
        """Extension: RMSNorm(q) -> RopeApply, RMSNorm(k) -> RopeApply and
        RMSNorm(v) (no weight) of one decode step in place, one launch
        (Gemma4TextInference.swift:352-381)."""

        def __init__(self, q, k_cache, v_cache, q_norm, k_norm, cos, sin, offset=0, position=None, eps=1e-6,
                     add_one_to_weight=False, norm_v=True):
            super().__init__(N.lib().pc_kernel_qk_norm_rope, _tc(q), _tc(k_cache), _tc(v_cache), _tc(q_norm),
                             _tc(k_norm), _tc(cos), _tc(sin), ctypes.c_float(eps), int(add_one_to_weight),
                             int(norm_v), int(offset), _tc(position),
                             keep=_keep(q, k_cache, v_cache, q_norm, k_norm, cos, sin, position))

    class QKVScatter(Kernel):
        """Extension: q and the new K/V rows out of one fused QKV Matmul."""

        def __init__(self, qkv, q_out, k_cache, v_cache, offset=0, position=None):
            super().__init__(N.lib().pc_kernel_qkv_scatter, _tc(qkv), _tc(q_out), _tc(k_cache), _tc(v_cache),
                             int(offset), _tc(position), keep=_keep(qkv, q_out, k_cache, v_cache, position))

    class GatedActivation(Kernel):
        """Extension: round(act(gate)) * up out of one fused gate/up Matmul."""
        GELU_TANH, SILU = 0, 1

        def __init__(self, gate_up, into, activation=0):
            super().__init__(N.lib().pc_kernel_gated_activation, _tc(gate_up), int(activation), _tc(into),
                             keep=_keep(gate_up, into))

    class AddRMSNorm(Kernel):
        """Extension: Add then RMSNorm; both results stored."""

        def __init__(self, a, b, norm_weight, sum_out, norm_out, eps=1e-6, add_one_to_weight=False):
            super().__init__(N.lib().pc_kernel_add_rmsnorm, _tc(a), _tc(b), _tc(norm_weight), ctypes.c_float(eps),
                             int(add_one_to_weight), _tc(sum_out), _tc(norm_out),
                             keep=_keep(a, b, norm_weight, sum_out, norm_out))


    class AllReduceAddRMSNorm(Kernel):
        """Extension: all-reduce (sum) of a PeerGroup partial buffer over peer
        memory, then Add(residual) and RMSNorm, in one kernel."""

        def __init__(self, group, buffer, residual, norm_weight, sum_out, norm_out, eps=1e-6,
                     add_one_to_weight=False):
            super().__init__(N.lib().pc_kernel_allreduce_add_rmsnorm, ctypes.byref(group.c), int(buffer),
                             _tc(residual), _tc(norm_weight), ctypes.c_float(eps), int(add_one_to_weight),
                             _tc(sum_out), _tc(norm_out), keep=_keep(group, residual, norm_weight, sum_out, norm_out))


class _MatmulAllReduceAddRMSNorm(Kernel):
    """Extension: Matmul (a . w^T, M <= 64, tensor cores) into this rank's
    PeerGroup partial buffer, then the all-reduce + Add + RMSNorm, in ONE
    kernel."""

    def __init__(self, a, w, group, buffer, residual, norm_weight, sum_out, norm_out, eps=1e-6,
                 add_one_to_weight=False):
        super().__init__(N.lib().pc_kernel_matmul_allreduce_add_rmsnorm, _tc(a), _tc(w), ctypes.byref(group.c),
                         int(buffer), _tc(residual), _tc(norm_weight), ctypes.c_float(eps), int(add_one_to_weight),
                         _tc(sum_out), _tc(norm_out), keep=_keep(a, w, group, residual, norm_weight, sum_out, norm_out))


Kernels.MatmulAllReduceAddRMSNorm = _MatmulAllReduceAddRMSNorm


class PeerGroup:
    """The tensor-parallel ranks' partial-sum buffers and control blocks,
    shared through CUDA IPC (one process per GPU on one node).

    Each rank allocates two [rows, cols] partial buffers of `dtype` and a
    zero-filled control block, and `all_gather(bytes) -> [bytes per rank]`
    (e.g. torch.distributed.all_gather_object) exchanges their IPC handles;
    the peers' buffers are then opened in this process. `partial(b)` is this
    rank's buffer b as a Tensor: the Matmul that produces the partial sum
    writes into it."""

    def __init__(self, device, world, rank, rows, cols, dtype, all_gather):
        if world > N.MAX_PEERS:
            raise PopcornError(PopcornError.tensorShapeMismatch, "at most %d ranks" % N.MAX_PEERS)
        L = N.lib()
        self.device, self.world, self.rank, self.rows, self.cols = device, world, rank, rows, cols
        self.dtype = DataType[dtype] if isinstance(dtype, str) else DataType(dtype)
        nbytes = rows * cols * L.pc_dtype_stride(int(self.dtype))
        own = []
        for _ in range(3):
            p = ctypes.c_void_p()
            _check(L.pc_buffer_alloc(device, nbytes if len(own) < 2 else 64, ctypes.byref(p)))
            own.append(p.value)
        zeros = (ctypes.c_uint8 * 64)()
        _check(L.pc_memcpy_htod_async(own[2], ctypes.cast(zeros, ctypes.c_void_p), 64, None))
        _check(L.pc_stream_synchronize(None))
        self._own = own
        handles = []
        for p in own:
            h = (ctypes.c_uint8 * 64)()
            _check(L.pc_ipc_get_handle(p, h))
            handles.append(bytes(h))
        gathered = all_gather(b"".join(handles))
        self._opened = []
        g = N.pc_peer_group()
        g.world, g.rank = world, rank
        for r in range(world):
            if r == rank:
                ptrs = own
            else:
                ptrs = []
                blob = gathered[r]
                for i in range(3):
                    h = (ctypes.c_uint8 * 64).from_buffer_copy(blob[64 * i:64 * (i + 1)])
                    p = ctypes.c_void_p()
                    _check(L.pc_ipc_open_handle(h, ctypes.byref(p)))
                    ptrs.append(p.value)
                    self._opened.append(p.value)
            g.partial[r][0] = ptrs[0]
            g.partial[r][1] = ptrs[1]
            g.control[r] = ctypes.cast(ptrs[2], ctypes.POINTER(ctypes.c_uint32))
        self.c = g

    def partial(self, b):
        return Tensor(self._own[b], (self.rows, self.cols), self.dtype, owner=self)

    def close(self):
        L = N.lib()
        for p in self._opened:
            L.pc_ipc_close_handle(p)
        self._opened = []


class DecodeStackKernel(Kernel):
    """Extension: a whole batch-1 decode step through a layer stack as one
    persistent kernel (pc_kernel_decode_stack). `desc` is a filled
    _native.pc_decode_stack_desc; `keep` holds the tensors it points into."""

    def __init__(self, desc, keep=()):
        self._desc = desc
        super().__init__(N.lib().pc_kernel_decode_stack, ctypes.byref(desc), keep=tuple(keep))

    @staticmethod
    def workspace_bytes(desc):
        out = ctypes.c_uint64()
        _check(N.lib().pc_decode_stack_workspace_bytes(ctypes.byref(desc), ctypes.byref(out)))
        return out.value


Kernels.DecodeStack = DecodeStackKernel


def device_error_check(device=0):
    """Reads and clears the device error word (bit 0: a bounded wait gave up)."""
    flags = ctypes.c_uint32()
    _check(N.lib().pc_device_error_check(device, ctypes.byref(flags)))
    return flags.value
