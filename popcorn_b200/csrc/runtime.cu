// runtime.cu — errors, tensors, KernelLibrary, KernelCommandEncoder and the
// non-kernel half of the C ABI.
#include <cstdio>
#include <cstring>
#include <sstream>

#include "launch.hpp"
#include "popcorn.hpp"

namespace popcorn {

namespace {
thread_local std::string g_last_error = "";
}

void set_last_error(const std::string& m) { g_last_error = m; }

[[noreturn]] void fail(int code, const std::string& message) { throw PopcornError{code, message}; }

// PopcornError.fromMetalError, PopcornError.swift:240-266, restated for CUDA.
void check_cuda(cudaError_t err, const char* what) {
    if (err == cudaSuccess) return;
    int code = PC_ERR_GPU_INTERNAL;
    switch (err) {
    case cudaErrorMemoryAllocation: code = PC_ERR_GPU_OUT_OF_MEMORY; break;
    case cudaErrorLaunchTimeout: code = PC_ERR_GPU_TIMEOUT; break;
    case cudaErrorIllegalAddress:
    case cudaErrorMisalignedAddress: code = PC_ERR_GPU_PAGE_FAULT; break;
    case cudaErrorInvalidResourceHandle:
    case cudaErrorInvalidDevicePointer:
    case cudaErrorInvalidValue: code = PC_ERR_GPU_INVALID_RESOURCE; break;
    case cudaErrorDevicesUnavailable:
    case cudaErrorNoDevice:
    case cudaErrorInvalidDevice: code = PC_ERR_GPU_DEVICE_REMOVED; break;
    case cudaErrorNotPermitted:
    case cudaErrorNotSupported: code = PC_ERR_GPU_ACCESS_REVOKED; break;
    default: break;
    }
    std::ostringstream os;
    os << what << ": " << cudaGetErrorName(err) << " (" << cudaGetErrorString(err) << ")";
    fail(code, os.str());
}

std::string dtype_name(int dtype) {
    static const char* names[] = {"u8", "u16", "u32", "u64", "i8", "i16", "i32", "i64", "f32", "f16", "bf16"};
    if (dtype < 0 || dtype > 10) return "unknown(" + std::to_string(dtype) + ")";
    return names[dtype];
}

// Tensor.DataType.stride, Tensor.swift:152-159.
int dtype_stride(int dtype) {
    switch (dtype) {
    case PC_U8: case PC_I8: return 1;
    case PC_U16: case PC_I16: case PC_F16: case PC_BF16: return 2;
    case PC_U32: case PC_I32: case PC_F32: return 4;
    case PC_U64: case PC_I64: return 8;
    default: return 0;
    }
}

std::string Tensor::shape_string() const {
    std::ostringstream os;
    os << "[";
    for (int i = 0; i < d.rank; ++i) os << (i ? ", " : "") << d.shape[i];
    os << "]";
    return os.str();
}

Tensor tensor_arg(const pc_tensor* t, const char* what) {
    if (!t) fail(PC_ERR_TENSOR_SHAPE_MISMATCH, std::string(what) + " tensor is null.");
    if (t->rank < 0 || t->rank > PC_MAX_RANK)
        fail(PC_ERR_TENSOR_INVALID_RANK, std::string(what) + " rank " + std::to_string(t->rank) +
                                             " is outside 0..8.");
    if (dtype_stride(t->dtype) == 0)
        fail(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION, std::string(what) + " has unknown data type " +
                                                           std::to_string(t->dtype) + ".");
    Tensor r(*t);
    for (int i = 0; i < t->rank; ++i)
        if (t->shape[i] < 0) fail(PC_ERR_TENSOR_SHAPE_MISMATCH, std::string(what) + " has a negative dimension.");
    if (r.element_count() > 0 && !t->data)
        fail(PC_ERR_TENSOR_SHAPE_MISMATCH, std::string(what) + " has no device buffer.");
    return r;
}

// ---- KernelLibrary ----------------------------------------------------------

std::vector<FunctionEntry>& function_registry() {
    static std::vector<FunctionEntry> registry;
    return registry;
}

RegisterFunctions::RegisterFunctions(std::initializer_list<FunctionEntry> entries) {
    auto& r = function_registry();
    r.insert(r.end(), entries.begin(), entries.end());
}

KernelLibrary::KernelLibrary(int device) : device_(device) {
    int count = 0;
    check_cuda(cudaGetDeviceCount(&count), "cudaGetDeviceCount");
    if (device < 0 || device >= count)
        fail(PC_ERR_GPU_DEVICE_REMOVED, "CUDA device " + std::to_string(device) + " does not exist (" +
                                            std::to_string(count) + " visible).");
    int major = 0, minor = 0;
    check_cuda(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device), "cudaDeviceGetAttribute");
    check_cuda(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device), "cudaDeviceGetAttribute");
    if (major != 10 || minor != 0)
        fail(PC_ERR_KERNEL_FUNCTION_NOT_FOUND, "this library holds sm_100a code only; device " + std::to_string(device) +
                                                   " is sm_" + std::to_string(major) + std::to_string(minor) + ".");
    sm_count_ = launch::device_info(device).sm_count;
    for (const auto& e : function_registry()) {
        if (table_.emplace(e.name, e.func).second) names_.push_back(e.name);
    }
}

const void* KernelLibrary::pipeline_state(const std::string& name) {
    std::lock_guard<std::mutex> guard(lock_);
    auto c = cache_.find(name);
    if (c != cache_.end()) return c->second;
    auto t = table_.find(name);
    if (t == table_.end()) fail(PC_ERR_KERNEL_FUNCTION_NOT_FOUND, "Kernel function '" + name + "' was not found.");
    // Make sure the function's image loads on this device (lazy loading).
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(device_);
    cudaFuncAttributes attr;
    cudaError_t err = cudaFuncGetAttributes(&attr, t->second);
    cudaSetDevice(prev);
    if (err != cudaSuccess) {
        cudaGetLastError();
        fail(PC_ERR_KERNEL_FUNCTION_NOT_FOUND, "Kernel function '" + name + "' cannot load on device " +
                                                   std::to_string(device_) + ": " + cudaGetErrorString(err));
    }
    cache_[name] = t->second;
    return t->second;
}

// ---- scratch ------------------------------------------------------------------

size_t ScratchSpec::byte_count() const {
    int64_t n = 1;
    for (auto s : shape) n *= s;
    int64_t b = n * dtype_stride(dtype);
    return size_t(b < 1 ? 1 : b);
}

// ---- KernelCommandEncoder -------------------------------------------------------

KernelCommandEncoder::KernelCommandEncoder(KernelLibrary& library, cudaStream_t stream,
                                           const pc_scratch_allocator* scratch)
    : library_(library), stream_(stream) {
    if (scratch) {
        scratch_ = *scratch;
        has_scratch_ = scratch->borrow != nullptr;
    }
}

void KernelCommandEncoder::encode(const Kernel& kernel) { kernel.encode(*this); }

// KernelCommandEncoder.swift:155-162: a barrier is needed on RAW, WAR and WAW.
bool KernelCommandEncoder::needs_barrier(const std::vector<Binding>& bindings) const {
    for (const auto& b : bindings) {
        auto it = access_by_buffer_.find(reinterpret_cast<uintptr_t>(b.tensor.data()));
        if (it == access_by_buffer_.end()) continue;
        int prev = it->second;
        if ((prev & PC_ACCESS_WRITE) && (b.access & PC_ACCESS_READ_WRITE)) return true;
        if ((b.access & PC_ACCESS_WRITE) && (prev & PC_ACCESS_READ_WRITE)) return true;
    }
    return false;
}

void KernelCommandEncoder::record_accesses(const std::vector<Binding>& bindings) {
    for (const auto& b : bindings) access_by_buffer_[reinterpret_cast<uintptr_t>(b.tensor.data())] |= b.access;
}

void KernelCommandEncoder::barrier() {
    // Launches on one stream are ordered; the barrier only resets the map.
    access_by_buffer_.clear();
    ++barriers_;
}

void KernelCommandEncoder::dispatch(const std::string& function_name, const std::vector<Binding>& bindings,
                                    const std::function<cudaError_t(cudaStream_t)>& launch) {
    if (needs_barrier(bindings)) barrier();
    library_.pipeline_state(function_name);
    int prev = 0;
    cudaGetDevice(&prev);
    if (prev != library_.device()) cudaSetDevice(library_.device());
    if (hook_) hook_(hook_ctx_, function_name.c_str(), PC_WILL_DISPATCH, stream_);
    cudaError_t err = launch(stream_);
    if (hook_) hook_(hook_ctx_, function_name.c_str(), PC_DID_DISPATCH, stream_);
    if (prev != library_.device()) cudaSetDevice(prev);
    check_cuda(err, function_name.c_str());
    ++dispatches_;
    record_accesses(bindings);
}

void KernelCommandEncoder::with_temporaries(const std::vector<ScratchSpec>& specs,
                                            const std::function<void(const std::vector<Tensor>&)>& body) {
    if (!has_scratch_)
        fail(PC_ERR_TENSOR_ALLOCATION_FAILED, "this kernel needs scratch memory but the encoder has no allocator.");
    std::vector<void*> borrowed;
    std::vector<Tensor> tensors;
    auto release_all = [&]() {
        for (auto it = borrowed.rbegin(); it != borrowed.rend(); ++it)
            if (scratch_.release) scratch_.release(scratch_.ctx, *it);
    };
    for (const auto& s : specs) {
        void* ptr = nullptr;
        int reused = 0;
        size_t len = s.byte_count();
        int st = scratch_.borrow(scratch_.ctx, len, &ptr, &reused);
        if (st != 0 || !ptr) {
            release_all();
            fail(st != 0 ? st : PC_ERR_TENSOR_ALLOCATION_FAILED,
                 "scratch allocator could not provide " + std::to_string(len) + " bytes.");
        }
        borrowed.push_back(ptr);
        // KernelCommandEncoder.swift:110: a reused buffer counts as written.
        if (reused) access_by_buffer_[reinterpret_cast<uintptr_t>(ptr)] = PC_ACCESS_WRITE;
        pc_tensor d{};
        d.data = ptr;
        d.dtype = s.dtype;
        d.rank = int32_t(s.shape.size());
        for (size_t i = 0; i < s.shape.size() && i < PC_MAX_RANK; ++i) d.shape[i] = s.shape[i];
        tensors.emplace_back(d);
    }
    try {
        body(tensors);
    } catch (...) {
        release_all();
        throw;
    }
    release_all();
}

}  // namespace popcorn

using namespace popcorn;

struct pc_library {
    KernelLibrary impl;
    explicit pc_library(int device) : impl(device) {}
};
struct pc_encoder {
    KernelCommandEncoder impl;
    pc_encoder(KernelLibrary& l, cudaStream_t s, const pc_scratch_allocator* a) : impl(l, s, a) {}
};

#define PC_GUARD_BEGIN try {
#define PC_GUARD_END                                  \
    }                                                 \
    catch (const PopcornError& e) {                   \
        set_last_error(e.message);                    \
        return e.code;                                \
    }                                                 \
    catch (const std::exception& e) {                 \
        set_last_error(e.what());                     \
        return PC_ERR_GPU_INTERNAL;                   \
    }                                                 \
    return PC_OK;

extern "C" {

const char* pc_last_error_message(void) { return g_last_error.c_str(); }

int pc_dtype_stride(int32_t dtype) { return dtype_stride(dtype); }

int64_t pc_scratch_spec_byte_count(const int64_t* shape, int32_t rank, int32_t dtype) {
    ScratchSpec s{std::vector<int64_t>(shape, shape + (rank > 0 ? rank : 0)), dtype};
    return int64_t(s.byte_count());
}

int pc_version(void) { return 10000; }

int pc_device_count(int* count) {
    PC_GUARD_BEGIN
    int c = 0;
    cudaError_t e = cudaGetDeviceCount(&c);
    if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver) {
        cudaGetLastError();
        c = 0;
    } else {
        check_cuda(e, "cudaGetDeviceCount");
    }
    *count = c;
    PC_GUARD_END
}

int pc_buffer_alloc(int device, size_t bytes, void** ptr) {
    PC_GUARD_BEGIN
    int prev = 0;
    cudaGetDevice(&prev);
    check_cuda(cudaSetDevice(device), "cudaSetDevice");
    cudaError_t e = cudaMalloc(ptr, bytes ? bytes : 1);
    cudaSetDevice(prev);
    if (e != cudaSuccess) {
        cudaGetLastError();
        fail(PC_ERR_TENSOR_ALLOCATION_FAILED, "cudaMalloc of " + std::to_string(bytes) + " bytes failed.");
    }
    PC_GUARD_END
}

int pc_ipc_get_handle(const void* ptr, uint8_t* handle64) {
    PC_GUARD_BEGIN
    if (!ptr || !handle64) fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "null pointer.");
    cudaIpcMemHandle_t h;
    check_cuda(cudaIpcGetMemHandle(&h, const_cast<void*>(ptr)), "cudaIpcGetMemHandle");
    static_assert(sizeof(h) == 64, "CUDA IPC handle size");
    memcpy(handle64, &h, 64);
    PC_GUARD_END
}

int pc_ipc_open_handle(const uint8_t* handle64, void** ptr) {
    PC_GUARD_BEGIN
    if (!ptr || !handle64) fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "null pointer.");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle64, 64);
    check_cuda(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
    PC_GUARD_END
}

int pc_ipc_close_handle(void* ptr) {
    PC_GUARD_BEGIN
    check_cuda(cudaIpcCloseMemHandle(ptr), "cudaIpcCloseMemHandle");
    PC_GUARD_END
}

int pc_buffer_free(void* ptr) {
    PC_GUARD_BEGIN
    check_cuda(cudaFree(ptr), "cudaFree");
    PC_GUARD_END
}

int pc_memcpy_htod_async(void* dst, const void* src, size_t bytes, void* stream) {
    PC_GUARD_BEGIN
    check_cuda(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, static_cast<cudaStream_t>(stream)),
               "cudaMemcpyAsync(H2D)");
    PC_GUARD_END
}

int pc_memcpy_dtoh_async(void* dst, const void* src, size_t bytes, void* stream) {
    PC_GUARD_BEGIN
    check_cuda(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, static_cast<cudaStream_t>(stream)),
               "cudaMemcpyAsync(D2H)");
    PC_GUARD_END
}

int pc_stream_synchronize(void* stream) {
    PC_GUARD_BEGIN
    check_cuda(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)), "cudaStreamSynchronize");
    PC_GUARD_END
}

int pc_library_create(int device, pc_library** out) {
    PC_GUARD_BEGIN
    *out = nullptr;
    *out = new pc_library(device);
    PC_GUARD_END
}

void pc_library_destroy(pc_library* library) { delete library; }

int pc_library_device(const pc_library* library, int* device) {
    PC_GUARD_BEGIN
    *device = library->impl.device();
    PC_GUARD_END
}

int pc_library_lookup(pc_library* library, const char* function_name, const void** handle) {
    PC_GUARD_BEGIN
    if (!function_name) fail(PC_ERR_KERNEL_FUNCTION_NOT_FOUND, "function name is null.");
    *handle = library->impl.pipeline_state(function_name);
    PC_GUARD_END
}

int pc_library_function_count(const pc_library* library) { return int(library->impl.names().size()); }

const char* pc_library_function_name(const pc_library* library, int index) {
    const auto& n = library->impl.names();
    if (index < 0 || size_t(index) >= n.size()) return nullptr;
    return n[size_t(index)].c_str();
}

int pc_encoder_create(pc_library* library, void* stream, const pc_scratch_allocator* scratch, pc_encoder** out) {
    PC_GUARD_BEGIN
    if (!library) fail(PC_ERR_KERNEL_FUNCTION_NOT_FOUND, "library is null.");
    *out = new pc_encoder(library->impl, static_cast<cudaStream_t>(stream), scratch);
    PC_GUARD_END
}

void pc_encoder_destroy(pc_encoder* encoder) { delete encoder; }

int pc_encoder_barrier(pc_encoder* encoder) {
    PC_GUARD_BEGIN
    encoder->impl.barrier();
    PC_GUARD_END
}

int64_t pc_encoder_barrier_count(const pc_encoder* encoder) { return encoder->impl.barrier_count(); }
int64_t pc_encoder_dispatch_count(const pc_encoder* encoder) { return encoder->impl.dispatch_count(); }

int pc_encoder_set_dispatch_hook(pc_encoder* encoder, pc_dispatch_hook hook, void* ctx) {
    PC_GUARD_BEGIN
    encoder->impl.set_hook(hook, ctx);
    PC_GUARD_END
}

int pc_encoder_stream(const pc_encoder* encoder, void** stream) {
    PC_GUARD_BEGIN
    *stream = encoder->impl.stream();
    PC_GUARD_END
}

}  // extern "C"

// Used by ops.cu for the kernel half of the ABI.
namespace popcorn {
KernelCommandEncoder& encoder_impl(pc_encoder* e) { return e->impl; }
}  // namespace popcorn
