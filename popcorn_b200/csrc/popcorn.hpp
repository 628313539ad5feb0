// popcorn.hpp — the C++ host layer behind the C ABI.
//
// Mirrors the reference's Swift surface type for type:
//   Tensor / Binding / Access        Sources/Popcorn/Tensor.swift:5-218
//   Kernel (value object)            Sources/Popcorn/Kernel.swift:15-70
//   KernelLibrary                    Sources/Popcorn/KernelLibrary.swift:4-41
//   KernelScratchAllocator           Sources/Popcorn/KernelResources.swift:5-36
//   KernelCommandEncoder             Sources/Popcorn/KernelCommandEncoder.swift:5-168
//   PopcornError                     Sources/Popcorn/PopcornError.swift:6-230
// The CUDA launchers the kernels call are declared in launch.hpp.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <functional>
#include <map>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/popcorn_cuda.h"

namespace popcorn {

struct PopcornError {
    int code;
    std::string message;
};

[[noreturn]] void fail(int code, const std::string& message);
// Maps a CUDA error to a PopcornError GPU code (-1013..-1019) and throws.
void check_cuda(cudaError_t err, const char* what);
std::string dtype_name(int dtype);
int dtype_stride(int dtype);

// ---- Tensor --------------------------------------------------------------

struct Tensor {
    pc_tensor d{};
    Tensor() = default;
    explicit Tensor(const pc_tensor& t) : d(t) {}
    int rank() const { return d.rank; }
    int dtype() const { return d.dtype; }
    void* data() const { return d.data; }
    int64_t operator[](int i) const { return d.shape[i]; }
    int64_t element_count() const {
        int64_t n = 1;
        for (int i = 0; i < d.rank; ++i) n *= d.shape[i];
        return n;
    }
    std::vector<int64_t> dims() const { return std::vector<int64_t>(d.shape, d.shape + d.rank); }
    bool same_shape(const Tensor& o) const { return dims() == o.dims(); }
    std::string shape_string() const;
};

// Validates a caller descriptor (rank range, known dtype, non-null data for
// non-empty tensors) and wraps it.
Tensor tensor_arg(const pc_tensor* t, const char* what);

struct Binding {
    Tensor tensor;
    int access;  // pc_access
};

// ---- KernelLibrary --------------------------------------------------------

struct FunctionEntry {
    const char* name;
    const void* func;  // __global__ function (host stub address)
};
// Each kernel translation unit contributes its functions to the table.
std::vector<FunctionEntry>& function_registry();
struct RegisterFunctions {
    RegisterFunctions(std::initializer_list<FunctionEntry> entries);
};

class KernelLibrary {
public:
    explicit KernelLibrary(int device);
    int device() const { return device_; }
    int sm_count() const { return sm_count_; }
    // KernelLibrary.pipelineState(for:): cached, thread-safe, -1006 if unknown.
    const void* pipeline_state(const std::string& name);
    const std::vector<std::string>& names() const { return names_; }

private:
    int device_;
    int sm_count_ = 148;
    std::mutex lock_;
    std::unordered_map<std::string, const void*> table_;
    std::unordered_map<std::string, const void*> cache_;
    std::vector<std::string> names_;
};

// ---- Scratch --------------------------------------------------------------

struct TemporaryBuffer {
    void* ptr;
    bool was_reused;
};

// ScratchSpec {shape, dataType}, ScratchSpec.swift:10-26.
struct ScratchSpec {
    std::vector<int64_t> shape;
    int dtype;
    size_t byte_count() const;
};

// ---- Encoder --------------------------------------------------------------

class Kernel;

class KernelCommandEncoder {
public:
    KernelCommandEncoder(KernelLibrary& library, cudaStream_t stream, const pc_scratch_allocator* scratch);
    KernelLibrary& library() { return library_; }
    cudaStream_t stream() const { return stream_; }
    int device() const { return library_.device(); }
    int sm_count() const { return library_.sm_count(); }

    void encode(const Kernel& kernel);
    // dispatch(_:), KernelCommandEncoder.swift:49-69: hazard check, library
    // lookup, hook, launch, record accesses.
    void dispatch(const std::string& function_name, const std::vector<Binding>& bindings,
                  const std::function<cudaError_t(cudaStream_t)>& launch);
    void barrier();

    // withTemporaryTensor, KernelCommandEncoder.swift:87-141: borrows one
    // buffer per spec from the caller's allocator for the body's duration.
    void with_temporaries(const std::vector<ScratchSpec>& specs,
                          const std::function<void(const std::vector<Tensor>&)>& body);

    bool has_scratch() const { return has_scratch_; }
    int64_t barrier_count() const { return barriers_; }
    int64_t dispatch_count() const { return dispatches_; }
    void set_hook(pc_dispatch_hook hook, void* ctx) { hook_ = hook; hook_ctx_ = ctx; }

private:
    bool needs_barrier(const std::vector<Binding>& bindings) const;
    void record_accesses(const std::vector<Binding>& bindings);

    KernelLibrary& library_;
    cudaStream_t stream_;
    pc_scratch_allocator scratch_{};
    bool has_scratch_ = false;
    std::unordered_map<uintptr_t, int> access_by_buffer_;
    int64_t barriers_ = 0;
    int64_t dispatches_ = 0;
    pc_dispatch_hook hook_ = nullptr;
    void* hook_ctx_ = nullptr;
};

// ---- Kernel ---------------------------------------------------------------

class Kernel {
public:
    virtual ~Kernel() = default;
    virtual const char* name() const = 0;
    // Kernel.tensors: the user-visible bindings.
    virtual std::vector<Binding> tensors() const = 0;
    virtual void encode(KernelCommandEncoder& encoder) const = 0;
    // The function names the kernel launches, ';'-separated.
    const std::string& function_names() const { return function_names_; }
    // L2 prefetch hint (slot 0 or 1) for kernels that stream from HBM; the
    // default rejects it.
    virtual void set_prefetch(int slot, const void* ptr, uint64_t bytes);
    // Scheduling hints (pc_kernel_hint); the default rejects them.
    virtual void set_hint(int hint, int64_t value);

protected:
    std::string function_names_;
};

}  // namespace popcorn
