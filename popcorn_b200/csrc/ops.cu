// ops.cu — the kernel value objects (validation + routing) and the kernel
// half of the C ABI. Each class restates one reference op's initialiser
// checks and routing; the arithmetic lives in the launchers (launch.hpp).
#include <memory>
#include <sstream>

#include "launch.hpp"
#include "popcorn.hpp"

namespace popcorn {
void set_last_error(const std::string& m);
KernelCommandEncoder& encoder_impl(pc_encoder* e);

void Kernel::set_prefetch(int, const void*, uint64_t) {
    fail(PC_ERR_KERNEL_FUNCTION_NOT_FOUND, std::string(name()) + " takes no L2 prefetch hint.");
}

void Kernel::set_hint(int hint, int64_t) {
    fail(PC_ERR_KERNEL_FUNCTION_NOT_FOUND, std::string(name()) + " takes no hint " + std::to_string(hint) + ".");
}

namespace {

void put_prefetch(launch::L2Prefetch& pf, int slot, const void* ptr, uint64_t bytes) {
    if (slot < 0 || slot > 1) fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "prefetch slot must be 0 or 1.");
    pf.ptr[slot] = bytes ? ptr : nullptr;
    pf.bytes[slot] = ptr ? bytes : 0;
}

std::string dims_string(const std::vector<int64_t>& v) {
    std::ostringstream os;
    os << "[";
    for (size_t i = 0; i < v.size(); ++i) os << (i ? ", " : "") << v[i];
    os << "]";
    return os.str();
}

void require_rank(const Tensor& t, int rank) {
    if (t.rank() != rank)
        fail(PC_ERR_TENSOR_INVALID_RANK, "Expected rank " + std::to_string(rank) + ", got " + std::to_string(t.rank()) + ".");
}

void require_elements(const Tensor& t, int64_t n, const char* what) {
    if (t.element_count() < n)
        fail(PC_ERR_TENSOR_SHAPE_MISMATCH, std::string(what) + " holds " + std::to_string(t.element_count()) +
                                               " elements; the dimensions need " + std::to_string(n) + ".");
}

bool is_float(int dt) { return dt == PC_F32 || dt == PC_F16 || dt == PC_BF16; }

const char* dt_tag(int dt) { return dt == PC_F32 ? "f32" : dt == PC_F16 ? "f16" : dt == PC_BF16 ? "bf16" : "x"; }

// ---------------------------------------------------------------------------
// Kernels.FlashAttention + _FlashDecoding (FlashAttention.swift:13-139,
// FlashDecoding.swift:6-90)
// ---------------------------------------------------------------------------
class FlashAttentionKernel : public Kernel {
public:
    FlashAttentionKernel(Tensor q, Tensor k, Tensor v, Tensor out, const Tensor* seq_lens, int64_t B, int64_t Nq,
                         int64_t Nkv, int64_t Sq, int64_t Sk, int64_t Hd, float scale, pc_attention_mask mask)
        : q_(q), k_(k), v_(v), out_(out), B_(B), Nq_(Nq), Nkv_(Nkv), Sq_(Sq), Sk_(Sk), Hd_(Hd), scale_(scale),
          mask_(mask) {
        if (seq_lens) {
            lens_ = *seq_lens;
            has_lens_ = true;
        }
        // FlashAttention.swift:27-36.
        if (Nkv <= 0 || Nq <= 0 || Nq % Nkv != 0)
            fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "FlashAttention query heads must be divisible by KV heads; got " +
                                                   std::to_string(Nq) + " and " + std::to_string(Nkv) + ".");
        if (Hd > 512)
            fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "FlashAttention head dim must be <= 512 (kernel limit); got " +
                                                   std::to_string(Hd) + ".");
        if (Hd <= 0 || B <= 0 || Sq <= 0)
            fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "FlashAttention needs batch, query length and head dim >= 1.");
        if (!has_lens_ && Sk <= 0)
            fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "FlashAttention needs at least one key (keyLen >= 1).");
        if (mask.kind < 0 || mask.kind > 2)
            fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "unknown attention mask kind " + std::to_string(mask.kind) + ".");
        if (mask.kind == PC_MASK_CAUSAL_SLIDING_WINDOW && mask.window < 1)
            fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "sliding-window length must be >= 1.");
        // _FDPartial / _FlashAttentionPlain dtype checks (FlashDecoding.swift:119-125, 199-205;
        // FlashAttention.swift:181-190), widened to f16 (extension).
        if (!is_float(q.dtype()) || !is_float(k.dtype()) || k.dtype() != v.dtype() || !is_float(out.dtype()))
            fail(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION,
                 "Unsupported FlashAttention data type combination: " + dtype_name(q.dtype()) + ", " +
                     dtype_name(k.dtype()) + ", " + dtype_name(v.dtype()) + ", " + dtype_name(out.dtype()) + ".");
        if (Sq == 1 && q.dtype() != k.dtype())
            fail(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION, "Unsupported FlashDecoding Q/K/V data type: " +
                                                               dtype_name(q.dtype()) + " with K/V " +
                                                               dtype_name(k.dtype()) + ".");
        require_elements(q, B * Nq * Sq * Hd, "FlashAttention q");
        require_elements(k, B * Nkv * Sk * Hd, "FlashAttention k");
        require_elements(v, B * Nkv * Sk * Hd, "FlashAttention v");
        require_elements(out, B * Nq * Sq * Hd, "FlashAttention out");
        if (has_lens_) {
            if (lens_.dtype() != PC_I32)
                fail(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION, "seq_lens must be i32; got " + dtype_name(lens_.dtype()) + ".");
            require_elements(lens_, B, "seq_lens");
        }
        path_ = pc_flash_attention_route(Sq, Hd, q.dtype());
        if (path_ == PC_PATH_DECODING) {
            function_names_ = std::string("flash_decoding_partial_") + dt_tag(k.dtype()) + ";flash_decoding_reduce_" +
                              dt_tag(out.dtype());
        } else {
            launch::FlashAttention fa = fa_params();
            path_ = launch::flash_attention_uses_tensor_cores(fa) ? PC_PATH_TENSOR : PC_PATH_PLAIN;
            function_names_ = path_ == PC_PATH_TENSOR ? "flash_attention_tc_bf16" : "flash_attention";
        }
    }

    const char* name() const override { return "FlashAttention"; }

    void set_prefetch(int slot, const void* ptr, uint64_t bytes) override {
        if (path_ != PC_PATH_DECODING) Kernel::set_prefetch(slot, ptr, bytes);
        put_prefetch(pf_, slot, ptr, bytes);
    }

    void set_hint(int hint, int64_t value) override {
        if (path_ != PC_PATH_DECODING || hint != PC_HINT_KV_EARLY) Kernel::set_hint(hint, value);
        kv_early_ = value ? 1 : 0;
    }

    std::vector<Binding> tensors() const override {
        std::vector<Binding> b = {{q_, PC_ACCESS_READ}, {k_, PC_ACCESS_READ}, {v_, PC_ACCESS_READ}, {out_, PC_ACCESS_WRITE}};
        if (has_lens_) b.push_back({lens_, PC_ACCESS_READ});
        return b;
    }

    launch::FlashAttention fa_params() const {
        return launch::FlashAttention{q_.data(), q_.dtype(), k_.data(), v_.data(), k_.dtype(), out_.data(), out_.dtype(),
                                      B_, Nq_, Nkv_, Sq_, Sk_, Hd_, scale_, mask_.kind, mask_.window};
    }

    void encode(KernelCommandEncoder& enc) const override {
        if (path_ != PC_PATH_DECODING) {
            launch::FlashAttention p = fa_params();
            enc.dispatch(path_ == PC_PATH_TENSOR ? "flash_attention_tc_bf16" : "flash_attention", tensors(),
                         [p](cudaStream_t s) { return launch::flash_attention(p, s); });
            return;
        }
        launch::FlashDecode p{q_.data(), q_.dtype(), k_.data(), v_.data(), k_.dtype(), out_.data(), out_.dtype(),
                              B_, Nq_, Nkv_, Sk_, Hd_, has_lens_ ? static_cast<const int32_t*>(lens_.data()) : nullptr,
                              scale_, mask_.kind, mask_.window, pf_, kv_early_};
        launch::FlashDecodePlan plan = launch::flash_decode_plan(p, enc.sm_count());
        // FlashDecoding.swift:55-59: partial O [B,Nq,P,Hd], m and l [B,Nq,P], f32.
        std::vector<ScratchSpec> specs = {{{B_, Nq_, plan.splits, Hd_}, PC_F32},
                                          {{B_, Nq_, plan.splits}, PC_F32},
                                          {{B_, Nq_, plan.splits}, PC_F32}};
        std::string partial_name = std::string("flash_decoding_partial_") + dt_tag(k_.dtype());
        std::string reduce_name = std::string("flash_decoding_reduce_") + dt_tag(out_.dtype());
        std::vector<Binding> reads = {{q_, PC_ACCESS_READ}, {k_, PC_ACCESS_READ}, {v_, PC_ACCESS_READ}};
        if (has_lens_) reads.push_back({lens_, PC_ACCESS_READ});
        enc.with_temporaries(specs, [&](const std::vector<Tensor>& t) {
            float* po = static_cast<float*>(t[0].data());
            float* pm = static_cast<float*>(t[1].data());
            float* pl = static_cast<float*>(t[2].data());
            std::vector<Binding> partial_b = reads;
            partial_b.push_back({t[0], PC_ACCESS_WRITE});
            partial_b.push_back({t[1], PC_ACCESS_WRITE});
            partial_b.push_back({t[2], PC_ACCESS_WRITE});
            std::vector<Binding> reduce_b = {{t[0], PC_ACCESS_READ}, {t[1], PC_ACCESS_READ}, {t[2], PC_ACCESS_READ},
                                             {out_, PC_ACCESS_WRITE}};
            if (plan.splits == 1) {
                // One split covers every key: the partial pass normalises
                // and writes the output itself.
                partial_b.push_back({out_, PC_ACCESS_WRITE});
            }
            enc.dispatch(partial_name, partial_b, [p, plan, po, pm, pl](cudaStream_t s) {
                return launch::flash_decode(p, plan, po, pm, pl, s);
            });
            if (plan.splits > 1)
                enc.dispatch(reduce_name, reduce_b, [p, plan, po, pm, pl](cudaStream_t s) {
                    return launch::flash_decode_combine(p, plan, po, pm, pl, s);
                });
        });
    }

private:
    Tensor q_, k_, v_, out_, lens_;
    bool has_lens_ = false;
    int64_t B_, Nq_, Nkv_, Sq_, Sk_, Hd_;
    float scale_;
    pc_attention_mask mask_;
    int path_ = PC_PATH_DECODING;
    launch::L2Prefetch pf_{};
    int kv_early_ = 0;
};

// ---------------------------------------------------------------------------
// Kernels.KVCacheWrite (KVCacheWrite.swift:5-72)
// ---------------------------------------------------------------------------
class KVCacheWriteKernel : public Kernel {
public:
    KVCacheWriteKernel(Tensor src, Tensor cache, int64_t B, int64_t Nkv, int64_t Snew, int64_t Smax, int64_t Hd,
                       int64_t offset)
        : src_(src), cache_(cache), p_{} {
        int s = src.dtype(), c = cache.dtype();
        // KVCacheWrite.swift:20-25 plus the f16 extension.
        if (s == PC_F32 && c == PC_F32) function_names_ = "kv_cache_write";
        else if (s == PC_BF16 && c == PC_BF16) function_names_ = "kv_cache_write_bf16";
        else if (s == PC_F32 && c == PC_BF16) function_names_ = "kv_cache_write_f32_to_bf16";
        else if (s == PC_F16 && c == PC_F16) function_names_ = "kv_cache_write_f16";
        else
            fail(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION, "Unsupported KV cache data type combination: " +
                                                               dtype_name(s) + ", " + dtype_name(c) + ".");
        if (offset < 0 || offset + Snew > Smax || B < 0 || Nkv < 0 || Snew < 0 || Hd < 0)
            fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "KV cache write range " + std::to_string(offset) + "..<" +
                                                   std::to_string(offset + Snew) + " exceeds cache length " +
                                                   std::to_string(Smax) + ".");
        require_elements(src, B * Nkv * Snew * Hd, "KVCacheWrite source");
        require_elements(cache, B * Nkv * Smax * Hd, "KVCacheWrite cache");
        p_ = launch::KVWrite{src.data(), s, cache.data(), c, B, Nkv, Snew, Smax, Hd, offset, nullptr};
    }
    const char* name() const override { return "KVCacheWrite"; }
    std::vector<Binding> tensors() const override { return {{src_, PC_ACCESS_READ}, {cache_, PC_ACCESS_WRITE}}; }
    void encode(KernelCommandEncoder& enc) const override {
        launch::KVWrite p = p_;
        enc.dispatch(function_names_, tensors(), [p](cudaStream_t s) { return launch::kv_cache_write(p, s); });
    }

private:
    Tensor src_, cache_;
    launch::KVWrite p_;
};

// ---------------------------------------------------------------------------
// Kernels.RMSNorm (RMSNorm.swift:7-96)
// ---------------------------------------------------------------------------
class RMSNormKernel : public Kernel {
public:
    RMSNormKernel(Tensor x, const Tensor* w, Tensor out, int64_t rows, int64_t H, float eps, bool add_one)
        : x_(x), out_(out) {
        int dt = x.dtype();
        if (dt == PC_F32) function_names_ = "rmsnorm";
        else if (dt == PC_F16) function_names_ = "rmsnorm_f16";
        else if (dt == PC_BF16) function_names_ = "rmsnorm_bf16";
        else fail(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION, "Unsupported RMSNorm data type: " + dtype_name(dt) + ".");
        // RMSNorm.metal:44-46: the output has x's type, the weight is f32.
        if (out.dtype() != dt)
            fail(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION, "RMSNorm output must be " + dtype_name(dt) + "; got " +
                                                               dtype_name(out.dtype()) + ".");
        if (w) {
            w_ = *w;
            has_w_ = true;
            if (w->dtype() != PC_F32)
                fail(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION, "RMSNorm weight must be f32; got " +
                                                                   dtype_name(w->dtype()) + ".");
            require_elements(*w, H, "RMSNorm weight");
        }
        if (H <= 0 || rows < 0) fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "RMSNorm hidden size must be >= 1.");
        require_elements(x, rows * H, "RMSNorm x");
        require_elements(out, rows * H, "RMSNorm out");
        p_ = launch::RMSNorm{x.data(), dt, has_w_ ? static_cast<const float*>(w->data()) : nullptr, out.data(),
                             out.dtype(), rows, H, eps, add_one ? 1 : 0};
    }
    const char* name() const override { return "RMSNorm"; }
    std::vector<Binding> tensors() const override {
        // With no weight the reference binds x in the weight slot (RMSNorm.swift:13).
        return {{x_, PC_ACCESS_READ}, {has_w_ ? w_ : x_, PC_ACCESS_READ}, {out_, PC_ACCESS_WRITE}};
    }
    void encode(KernelCommandEncoder& enc) const override {
        launch::RMSNorm p = p_;
        enc.dispatch(function_names_, tensors(), [p](cudaStream_t s) { return launch::rmsnorm(p, s); });
    }

private:
    Tensor x_, w_, out_;
    bool has_w_ = false;
    launch::RMSNorm p_{};
};

// Dtype combinations the matvec serves: Matmul.swift:362-374
// (fff, f.bf.f, bf.bf.f, bf.bf.bf) plus the f16 forms (MPPMatvec's
// f16.f16.f16, f16.f16.f32) and f32.f16.f32 (Matvec.metal:130).
bool matvec_dtypes_ok(int x, int w, int o) {
    if (x == PC_F32 && w == PC_F32 && o == PC_F32) return true;
    if (w != PC_BF16 && w != PC_F16) return false;
    return (x == PC_F32 || x == w) && (o == PC_F32 || o == w);
}

// ---------------------------------------------------------------------------
// Kernels.Matmul (Matmul.swift:9-93, 233-277)
// ---------------------------------------------------------------------------
class MatmulKernel : public Kernel {
public:
    MatmulKernel(Tensor a, Tensor b, Tensor c, int64_t m, int64_t k, int64_t n, bool transpose_b)
        : a_(a), b_(b), c_(c), m_(m), k_(k), n_(n), tb_(transpose_b) {
        int ad = a.dtype(), bd = b.dtype(), cd = c.dtype();
        if (m < 0 || k < 0 || n < 0) fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "Matmul dimensions must be >= 0.");
        require_elements(a, m * k, "Matmul A");
        require_elements(b, k * n, "Matmul B");
        require_elements(c, m * n, "Matmul C");
        gemv_ = (m == 1 && transpose_b && matvec_dtypes_ok(ad, bd, cd));
        if (gemv_) {
            function_names_ = std::string("matvec_nk_") + dt_tag(ad) + "_" + dt_tag(bd) + "_" + dt_tag(cd);
            return;
        }
        // Matmul.swift:198-231 (naive / MPP combinations) plus f16.
        bool ok = (ad == PC_F32 && bd == PC_F32 && cd == PC_F32) ||
                  (ad == PC_F32 && (bd == PC_F16 || bd == PC_BF16) && cd == PC_F32) ||
                  ((ad == PC_BF16 || ad == PC_F16) && bd == ad && (cd == PC_F32 || cd == ad));
        if (!ok)
            fail(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION, "Unsupported matmul data type combination: " +
                                                               dtype_name(ad) + ", " + dtype_name(bd) + ", " +
                                                               dtype_name(cd) + ".");
        launch::Matmul p = params();
        if (m <= 64 && launch::matmul_uses_tensor_cores(p))
            ctr_base_ = launch::gemm_reserve_counters(2 * ((n + 127) / 128));  // >= the split-K tile count
        function_names_ = !launch::matmul_uses_tensor_cores(p) ? "matmul"
                          : p.transpose_b                       ? "matmul_tc_bf16_tb"
                                                                : "matmul_tc_bf16_nn";
    }
    launch::Matmul params() const {
        launch::Matmul p{a_.data(), a_.dtype(), b_.data(), b_.dtype(), c_.data(), c_.dtype(), m_, k_, n_, tb_ ? 1 : 0};
        p.ctr_base = ctr_base_;
        return p;
    }
    const char* name() const override { return "Matmul"; }
    void set_prefetch(int slot, const void* ptr, uint64_t bytes) override {
        if (!gemv_) Kernel::set_prefetch(slot, ptr, bytes);
        put_prefetch(pf_, slot, ptr, bytes);
    }
    std::vector<Binding> tensors() const override {
        return {{a_, PC_ACCESS_READ}, {b_, PC_ACCESS_READ}, {c_, PC_ACCESS_WRITE}};
    }
    void encode(KernelCommandEncoder& enc) const override {
        if (m_ == 0 || n_ == 0) return;
        if (gemv_) {
            launch::Gemv g{};
            g.x = a_.data(); g.x_dtype = a_.dtype(); g.w = b_.data(); g.w_dtype = b_.dtype();
            g.out = c_.data(); g.out_dtype = c_.dtype(); g.K = k_; g.N = n_;
            g.epilogue = launch::Epilogue::kStore;
            g.pf = pf_;
            enc.dispatch(function_names_, tensors(), [g](cudaStream_t s) { return launch::gemv(g, s); });
            return;
        }
        launch::Matmul p = params();
        // (an encoder without a scratch allocator runs the unsplit GEMM)
        const size_t ws =
            enc.has_scratch() && launch::matmul_uses_tensor_cores(p) ? launch::matmul_tcgen05_workspace(p) : 0;
        if (ws == 0) {
            enc.dispatch(function_names_, tensors(), [p](cudaStream_t s) { return launch::matmul(p, s); });
            return;
        }
        // split-K partials of a skinny tensor-core GEMM come from the scratch allocator
        std::vector<ScratchSpec> specs = {{{int64_t(ws)}, PC_U8}};
        enc.with_temporaries(specs, [&](const std::vector<Tensor>& t) {
            launch::Matmul q = p;
            q.workspace = t[0].data();
            std::vector<Binding> b = tensors();
            b.push_back({t[0], PC_ACCESS_READ_WRITE});
            enc.dispatch(function_names_, b, [q](cudaStream_t s) { return launch::matmul(q, s); });
        });
    }

private:
    Tensor a_, b_, c_;
    int64_t m_, k_, n_;
    bool tb_;
    bool gemv_ = false;
    launch::L2Prefetch pf_{};
    int ctr_base_ = -1;
};

// ---------------------------------------------------------------------------
// Elementwise: GeluTanh, SiLU, Mul, Add (GeluTanh.swift, Mul.swift, Add.swift)
// ---------------------------------------------------------------------------
class UnaryKernel : public Kernel {
public:
    UnaryKernel(launch::Unary op, Tensor x, Tensor out, float scalar = 1.0f)
        : op_(op), x_(x), out_(out), scalar_(scalar) {
        const char* base = op == launch::Unary::kGeluTanh ? "gelu_tanh" : op == launch::Unary::kSilu ? "silu" : "scalar_mul";
        const char* opname = op == launch::Unary::kGeluTanh ? "GeluTanh" : op == launch::Unary::kSilu ? "SiLU" : "ScalarMul";
        if (!x.same_shape(out))
            fail(PC_ERR_TENSOR_SHAPE_MISMATCH, std::string(opname) + " output shape must match input; got " +
                                                   out.shape_string() + ", expected " + x.shape_string() + ".");
        if (!is_float(x.dtype()) || out.dtype() != x.dtype())
            fail(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION, std::string("Unsupported ") + opname + " data type: " +
                                                               dtype_name(x.dtype()) + ".");
        function_names_ = x.dtype() == PC_F32 ? std::string(base) : std::string(base) + "_" + dt_tag(x.dtype());
        name_ = opname;
    }
    const char* name() const override { return name_; }
    std::vector<Binding> tensors() const override { return {{x_, PC_ACCESS_READ}, {out_, PC_ACCESS_WRITE}}; }
    void encode(KernelCommandEncoder& enc) const override {
        auto op = op_;
        const void* x = x_.data();
        void* o = out_.data();
        int dt = x_.dtype();
        int64_t n = x_.element_count();
        if (n == 0) return;
        const float sc = scalar_;
        enc.dispatch(function_names_, tensors(),
                     [=](cudaStream_t s) { return launch::unary(op, x, dt, o, dt, n, s, sc); });
    }

private:
    launch::Unary op_;
    Tensor x_, out_;
    float scalar_;
    const char* name_;
};

// Kernels.AttentionMaskBuild(mask:slidingWindow:) (AttentionMaskBuild.swift)
class AttentionMaskBuildKernel : public Kernel {
public:
    AttentionMaskBuildKernel(Tensor mask, int32_t window) : mask_(mask), window_(window) {
        if (mask.rank() != 2)
            fail(PC_ERR_TENSOR_INVALID_RANK, "expected rank 2, got rank " + std::to_string(mask.rank()) + ".");
        if (mask.dtype() != PC_F32) fail(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION, "the attention mask is f32.");
        function_names_ = "attention_mask_build";
    }
    const char* name() const override { return "AttentionMaskBuild"; }
    std::vector<Binding> tensors() const override { return {{mask_, PC_ACCESS_WRITE}}; }
    void encode(KernelCommandEncoder& enc) const override {
        float* m = static_cast<float*>(mask_.data());
        const int64_t sq = mask_[0], sk = mask_[1];
        const int32_t w = window_;
        enc.dispatch(function_names_, tensors(),
                     [=](cudaStream_t s) { return launch::attention_mask_build(m, sq, sk, w, s); });
    }

private:
    Tensor mask_;
    int32_t window_;
};

class BinaryKernel : public Kernel {
public:
    BinaryKernel(launch::Binary op, Tensor a, Tensor b, Tensor out) : op_(op), a_(a), b_(b), out_(out) {
        const char* base = op == launch::Binary::kMul ? "mul" : "add";
        name_ = op == launch::Binary::kMul ? "Mul" : "Add";
        if (!a.same_shape(b) || !a.same_shape(out))
            fail(PC_ERR_TENSOR_SHAPE_MISMATCH, std::string(name_) + " shapes must match; got " + a.shape_string() +
                                                   ", " + b.shape_string() + ", " + out.shape_string() + ".");
        if (!is_float(a.dtype()) || b.dtype() != a.dtype() || out.dtype() != a.dtype())
            fail(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION, std::string("Unsupported ") + name_ + " data type: " +
                                                               dtype_name(a.dtype()) + ".");
        function_names_ = a.dtype() == PC_F32 ? std::string(base) : std::string(base) + "_" + dt_tag(a.dtype());
    }
    const char* name() const override { return name_; }
    std::vector<Binding> tensors() const override {
        return {{a_, PC_ACCESS_READ}, {b_, PC_ACCESS_READ}, {out_, PC_ACCESS_WRITE}};
    }
    void encode(KernelCommandEncoder& enc) const override {
        auto op = op_;
        const void* a = a_.data();
        const void* b = b_.data();
        void* o = out_.data();
        int dt = a_.dtype();
        int64_t n = a_.element_count();
        if (n == 0) return;
        enc.dispatch(function_names_, tensors(), [=](cudaStream_t s) { return launch::binary(op, a, b, o, dt, n, s); });
    }

private:
    launch::Binary op_;
    Tensor a_, b_, out_;
    const char* name_;
};

// ---------------------------------------------------------------------------
// Fused decode ops (extensions)
// ---------------------------------------------------------------------------
void check_norm_weight(const Tensor* w, int64_t K) {
    if (!w) return;
    if (w->dtype() != PC_F32)
        fail(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION, "RMSNorm weight must be f32; got " + dtype_name(w->dtype()) + ".");
    require_elements(*w, K, "RMSNorm weight");
}

void check_row_vector(const Tensor& x, int64_t K, const char* what) {
    if (x.element_count() != K)
        fail(PC_ERR_TENSOR_SHAPE_MISMATCH, std::string(what) + " must hold one row of " + std::to_string(K) +
                                               " elements; got " + x.shape_string() + ".");
}

class FusedGemvKernel : public Kernel {
public:
    FusedGemvKernel(const char* name, std::vector<Binding> bindings, launch::Gemv g, std::string fn)
        : name_(name), bindings_(std::move(bindings)), g_(g) {
        function_names_ = std::move(fn);
    }
    const char* name() const override { return name_; }
    std::vector<Binding> tensors() const override { return bindings_; }
    void set_prefetch(int slot, const void* ptr, uint64_t bytes) override { put_prefetch(g_.pf, slot, ptr, bytes); }
    void encode(KernelCommandEncoder& enc) const override {
        launch::Gemv g = g_;
        enc.dispatch(function_names_, bindings_, [g](cudaStream_t s) { return launch::gemv(g, s); });
    }

private:
    const char* name_;
    std::vector<Binding> bindings_;
    launch::Gemv g_;
};

std::unique_ptr<Kernel> make_rmsnorm_matmul(const Tensor& x, const Tensor* nw, float eps, bool add_one, const Tensor& w,
                                            const Tensor& out) {
    require_rank(w, 2);
    int64_t N = w[0], K = w[1];
    check_row_vector(x, K, "RMSNorm+Matmul x");
    check_row_vector(out, N, "RMSNorm+Matmul out");
    check_norm_weight(nw, K);
    if (!is_float(x.dtype()) || w.dtype() != x.dtype() || out.dtype() != x.dtype() || x.dtype() == PC_F32)
        fail(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION, "RMSNorm+Matmul needs x, w and out all f16 or all bf16.");
    launch::Gemv g{};
    g.x = x.data(); g.x_dtype = x.dtype(); g.w = w.data(); g.w_dtype = w.dtype(); g.out = out.data();
    g.out_dtype = out.dtype(); g.K = K; g.N = N; g.has_norm = true;
    g.norm_weight = nw ? static_cast<const float*>(nw->data()) : nullptr; g.eps = eps; g.add_one = add_one;
    g.epilogue = launch::Epilogue::kStore;
    std::vector<Binding> b = {{x, PC_ACCESS_READ}, {w, PC_ACCESS_READ}, {out, PC_ACCESS_WRITE}};
    if (nw) b.push_back({*nw, PC_ACCESS_READ});
    return std::make_unique<FusedGemvKernel>("RMSNormMatmul", b, g, std::string("rmsnorm_matvec_") + dt_tag(x.dtype()));
}

std::unique_ptr<Kernel> make_gated_mlp(const Tensor& x, const Tensor* nw, float eps, bool add_one, const Tensor& wg,
                                       const Tensor& wu, int act, const Tensor& out) {
    require_rank(wg, 2);
    require_rank(wu, 2);
    if (wg.dims() != wu.dims())
        fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "gate and up weights must have the same shape; got " + wg.shape_string() +
                                               " and " + wu.shape_string() + ".");
    int64_t F = wg[0], K = wg[1];
    check_row_vector(x, K, "GatedMLP x");
    check_row_vector(out, F, "GatedMLP out");
    check_norm_weight(nw, K);
    if (act != PC_ACT_GELU_TANH && act != PC_ACT_SILU)
        fail(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION, "unknown activation " + std::to_string(act) + ".");
    int dt = x.dtype();
    if ((dt != PC_F16 && dt != PC_BF16) || wg.dtype() != dt || wu.dtype() != dt || out.dtype() != dt)
        fail(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION, "GatedMLP needs x, weights and out all f16 or all bf16.");
    launch::Gemv g{};
    g.x = x.data(); g.x_dtype = dt; g.w = wg.data(); g.w2 = wu.data(); g.w_dtype = dt; g.out = out.data();
    g.out_dtype = dt; g.K = K; g.N = F; g.has_norm = nw != nullptr;
    g.norm_weight = nw ? static_cast<const float*>(nw->data()) : nullptr; g.eps = eps; g.add_one = add_one;
    g.epilogue = launch::Epilogue::kGated; g.activation = act;
    std::vector<Binding> b = {{x, PC_ACCESS_READ}, {wg, PC_ACCESS_READ}, {wu, PC_ACCESS_READ}, {out, PC_ACCESS_WRITE}};
    if (nw) b.push_back({*nw, PC_ACCESS_READ});
    return std::make_unique<FusedGemvKernel>("GatedMLP", b, g,
                                             std::string(act == PC_ACT_SILU ? "swiglu_matvec_" : "geglu_matvec_") + dt_tag(dt));
}

std::unique_ptr<Kernel> make_matmul_residual(const Tensor& a, const Tensor& w, const Tensor& res, const Tensor& out) {
    require_rank(w, 2);
    int64_t N = w[0], K = w[1];
    check_row_vector(a, K, "Matmul+Add a");
    check_row_vector(res, N, "Matmul+Add residual");
    check_row_vector(out, N, "Matmul+Add out");
    int dt = a.dtype();
    if ((dt != PC_F16 && dt != PC_BF16) || w.dtype() != dt || res.dtype() != dt || out.dtype() != dt)
        fail(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION, "Matmul+Add needs all tensors f16 or all bf16.");
    launch::Gemv g{};
    g.x = a.data(); g.x_dtype = dt; g.w = w.data(); g.w_dtype = dt; g.out = out.data(); g.out_dtype = dt;
    g.K = K; g.N = N; g.epilogue = launch::Epilogue::kResidual; g.residual = res.data();
    std::vector<Binding> b = {{a, PC_ACCESS_READ}, {w, PC_ACCESS_READ}, {res, PC_ACCESS_READ}, {out, PC_ACCESS_WRITE}};
    return std::make_unique<FusedGemvKernel>("MatmulResidual", b, g, std::string("matvec_residual_") + dt_tag(dt));
}

std::unique_ptr<Kernel> make_qkv(const Tensor& x, const Tensor* nw, float eps, bool add_one, const Tensor& wqkv,
                                 const Tensor& q_out, const Tensor& kc, const Tensor& vc, int64_t offset,
                                 const Tensor* pos) {
    require_rank(wqkv, 2);
    require_rank(kc, 4);
    require_rank(q_out, 4);
    if (!kc.same_shape(vc))
        fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "K and V caches must have the same shape; got " + kc.shape_string() + " and " +
                                               vc.shape_string() + ".");
    int64_t K = wqkv[1];
    int64_t Nkv = kc[1], Smax = kc[2], Hd = kc[3];
    int64_t Nq = q_out[1];
    if (kc[0] != 1 || q_out[0] != 1 || q_out[2] != 1 || q_out[3] != Hd)
        fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "QKV projection is for batch 1, one token: q_out [1,Nq,1,Hd], caches [1,Nkv,Smax,Hd].");
    if (wqkv[0] != (Nq + 2 * Nkv) * Hd)
        fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "w_qkv must have (Nq + 2*Nkv)*Hd = " + std::to_string((Nq + 2 * Nkv) * Hd) +
                                               " rows; got " + std::to_string(wqkv[0]) + ".");
    check_row_vector(x, K, "QKV x");
    check_norm_weight(nw, K);
    if (!pos && (offset < 0 || offset >= Smax))
        fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "KV cache write range " + std::to_string(offset) + "..<" +
                                               std::to_string(offset + 1) + " exceeds cache length " + std::to_string(Smax) + ".");
    if (pos && (pos->dtype() != PC_I32 || pos->element_count() < 1))
        fail(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION, "position must be an i32 tensor with one element.");
    int dt = x.dtype();
    if ((dt != PC_F16 && dt != PC_BF16) || wqkv.dtype() != dt || q_out.dtype() != dt || kc.dtype() != dt || vc.dtype() != dt)
        fail(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION, "QKV projection needs all tensors f16 or all bf16.");
    launch::Gemv g{};
    g.x = x.data(); g.x_dtype = dt; g.w = wqkv.data(); g.w_dtype = dt; g.out = q_out.data(); g.out_dtype = dt;
    g.K = K; g.N = wqkv[0]; g.has_norm = true; g.norm_weight = nw ? static_cast<const float*>(nw->data()) : nullptr;
    g.eps = eps; g.add_one = add_one; g.epilogue = launch::Epilogue::kQKV;
    g.k_cache = kc.data(); g.v_cache = vc.data(); g.q_rows = Nq * Hd; g.kv_rows = Nkv * Hd; g.Hd = Hd; g.Smax = Smax;
    g.offset = offset; g.pos_dev = pos ? static_cast<const int32_t*>(pos->data()) : nullptr;
    std::vector<Binding> b = {{x, PC_ACCESS_READ}, {wqkv, PC_ACCESS_READ}, {q_out, PC_ACCESS_WRITE},
                              {kc, PC_ACCESS_WRITE}, {vc, PC_ACCESS_WRITE}};
    if (nw) b.push_back({*nw, PC_ACCESS_READ});
    if (pos) b.push_back({*pos, PC_ACCESS_READ});
    return std::make_unique<FusedGemvKernel>("QKVProjection", b, g, std::string("qkv_matvec_") + dt_tag(dt));
}

// ---------------------------------------------------------------------------
// Kernels.Argmax (Argmax.swift)
// ---------------------------------------------------------------------------
class ArgmaxKernel : public Kernel {
public:
    ArgmaxKernel(Tensor x, Tensor idx, int axis) : x_(x), idx_(idx) {
        const int rank = x.rank();
        const int ax = axis < 0 ? rank + axis : axis;
        // Argmax.swift:25-29
        if (rank < 1 || ax != rank - 1)
            fail(PC_ERR_TENSOR_INVALID_AXIS, "Argmax axis " + std::to_string(axis) + " is invalid for rank " +
                                                 std::to_string(rank) + ".");
        if (!is_float(x.dtype()))
            fail(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION, "Argmax input must be f32 (f16 / bf16 extension).");
        if (idx.dtype() != PC_I32) fail(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION, "Argmax indices must be int32.");
        const int64_t N = x[ax];
        const int64_t rows = N > 0 ? x.element_count() / N : 0;
        // Argmax.swift:31-35
        if (idx.element_count() != rows)
            fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "Argmax indices must contain " + std::to_string(rows) +
                                                   " elements; got " + std::to_string(idx.element_count()) + ".");
        if (N > int64_t(0x7fffffff)) fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "Argmax row longer than int32 indices.");
        p_ = launch::Argmax{x.data(), x.dtype(), static_cast<int32_t*>(idx.data()), rows, N, 1, N, nullptr, nullptr};
        function_names_ = N < 32 ? "argmax" : "argmax_row";  // Argmax.swift:21
    }
    const char* name() const override { return "Argmax"; }
    std::vector<Binding> tensors() const override { return {{x_, PC_ACCESS_READ}, {idx_, PC_ACCESS_WRITE}}; }
    void encode(KernelCommandEncoder& enc) const override {
        launch::Argmax p = p_;
        if (p.N >= 32 && enc.has_scratch()) launch::argmax_plan(p, enc.sm_count());
        if (p.chunks <= 1) {
            enc.dispatch(function_names_, tensors(), [p](cudaStream_t s) { return launch::argmax(p, s); });
            return;
        }
        std::vector<ScratchSpec> specs = {{{p.rows * p.chunks}, PC_F32}, {{p.rows * p.chunks}, PC_I32}};
        enc.with_temporaries(specs, [&](const std::vector<Tensor>& t) {
            launch::Argmax q = p;
            q.part_v = static_cast<float*>(t[0].data());
            q.part_i = static_cast<int32_t*>(t[1].data());
            std::vector<Binding> b = tensors();
            b.push_back({t[0], PC_ACCESS_READ_WRITE});
            b.push_back({t[1], PC_ACCESS_READ_WRITE});
            enc.dispatch(function_names_, b, [q](cudaStream_t s) { return launch::argmax(q, s); });
        });
    }

private:
    Tensor x_, idx_;
    launch::Argmax p_{};
};

// ---------------------------------------------------------------------------
// Batched-decode helpers (batched.cu)
// ---------------------------------------------------------------------------
inline bool aligned16_ptr(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

class QKVScatterKernel : public Kernel {
public:
    QKVScatterKernel(Tensor qkv, Tensor q, Tensor kc, Tensor vc, int64_t offset, const Tensor* pos)
        : qkv_(qkv), q_(q), kc_(kc), vc_(vc) {
        const int dt = qkv.dtype();
        if (!is_float(dt) || q.dtype() != dt || kc.dtype() != dt || vc.dtype() != dt)
            fail(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION, "QKVScatter needs one float dtype for qkv, q and caches.");
        if (qkv.rank() != 2 || q.rank() != 4 || kc.rank() != 4 || !kc.same_shape(vc))
            fail(PC_ERR_TENSOR_INVALID_RANK, "QKVScatter wants qkv [B,(Nq+2Nkv)*Hd], q [B,Nq,1,Hd], caches [B,Nkv,Smax,Hd].");
        const int64_t B = q[0], Nq = q[1], Hd = q[3], Nkv = kc[1], Smax = kc[2];
        if (q[2] != 1 || kc[0] != B || kc[3] != Hd || qkv[0] != B || qkv[1] != (Nq + 2 * Nkv) * Hd)
            fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "QKVScatter shapes disagree: qkv " + qkv.shape_string() + ", q " +
                                                   q.shape_string() + ", cache " + kc.shape_string() + ".");
        const int es = dtype_stride(dt);
        if ((Hd * es) % 16 != 0 || !aligned16_ptr(qkv.data()) || !aligned16_ptr(q.data()) ||
            !aligned16_ptr(kc.data()) || !aligned16_ptr(vc.data()))
            fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "QKVScatter needs Hd rows of a multiple of 16 bytes, 16-byte aligned.");
        if (!pos && (offset < 0 || offset >= Smax))
            fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "KV cache write offset " + std::to_string(offset) +
                                                   " outside cache length " + std::to_string(Smax) + ".");
        if (pos) {
            if (pos->dtype() != PC_I32 || pos->element_count() < 1)
                fail(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION, "position must be int32 [1].");
            pos_ = *pos;
            has_pos_ = true;
        }
        p_ = launch::QKVScatter{qkv.data(), q.data(), kc.data(), vc.data(), dt, B, Nq, Nkv, Hd, Smax, offset,
                                pos ? static_cast<const int32_t*>(pos->data()) : nullptr};
        function_names_ = "qkv_scatter";
    }
    const char* name() const override { return "QKVScatter"; }
    std::vector<Binding> tensors() const override {
        std::vector<Binding> b = {{qkv_, PC_ACCESS_READ}, {q_, PC_ACCESS_WRITE}, {kc_, PC_ACCESS_WRITE},
                                  {vc_, PC_ACCESS_WRITE}};
        if (has_pos_) b.push_back({pos_, PC_ACCESS_READ});
        return b;
    }
    void encode(KernelCommandEncoder& enc) const override {
        launch::QKVScatter p = p_;
        enc.dispatch(function_names_, tensors(), [p](cudaStream_t s) { return launch::qkv_scatter(p, s); });
    }

private:
    Tensor qkv_, q_, kc_, vc_, pos_;
    bool has_pos_ = false;
    launch::QKVScatter p_{};
};

class GatedActivationKernel : public Kernel {
public:
    GatedActivationKernel(Tensor gu, int act, Tensor out) : gu_(gu), out_(out), act_(act) {
        const int dt = gu.dtype();
        if (!is_float(dt) || out.dtype() != dt)
            fail(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION, "GatedActivation needs one float dtype.");
        if (act != PC_ACT_GELU_TANH && act != PC_ACT_SILU)
            fail(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION, "unknown activation.");
        if (gu.rank() != 2 || out.rank() != 2 || out[0] != gu[0] || gu[1] != 2 * out[1])
            fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "GatedActivation wants gate_up [rows,2F] and out [rows,F]; got " +
                                                   gu.shape_string() + ", " + out.shape_string() + ".");
        rows_ = out[0];
        F_ = out[1];
        function_names_ = dt == PC_F32 ? "gated_activation" : std::string("gated_activation_") + dt_tag(dt);
    }
    const char* name() const override { return "GatedActivation"; }
    std::vector<Binding> tensors() const override { return {{gu_, PC_ACCESS_READ}, {out_, PC_ACCESS_WRITE}}; }
    void encode(KernelCommandEncoder& enc) const override {
        const void* gu = gu_.data();
        void* o = out_.data();
        const int dt = gu_.dtype(), act = act_;
        const int64_t rows = rows_, F = F_;
        enc.dispatch(function_names_, tensors(),
                     [=](cudaStream_t s) { return launch::gated_activation(gu, o, dt, rows, F, act, s); });
    }

private:
    Tensor gu_, out_;
    int act_;
    int64_t rows_ = 0, F_ = 0;
};

class AddRMSNormKernel : public Kernel {
public:
    AddRMSNormKernel(Tensor a, Tensor b, const Tensor* w, float eps, bool add_one, Tensor sum, Tensor norm)
        : a_(a), b_(b), sum_(sum), norm_(norm) {
        const int dt = a.dtype();
        if (!is_float(dt) || b.dtype() != dt || sum.dtype() != dt || norm.dtype() != dt)
            fail(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION, "AddRMSNorm needs one float dtype.");
        if (!a.same_shape(b) || !a.same_shape(sum) || !a.same_shape(norm) || a.rank() < 1)
            fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "AddRMSNorm shapes must match; got " + a.shape_string() + ", " +
                                                   b.shape_string() + ".");
        const int64_t H = a[a.rank() - 1];
        if (H <= 0) fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "AddRMSNorm hidden size must be >= 1.");
        if (w) {
            if (w->dtype() != PC_F32)
                fail(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION, "RMSNorm weight must be f32.");
            require_elements(*w, H, "AddRMSNorm weight");
            w_ = *w;
            has_w_ = true;
        }
        p_ = launch::AddRMSNorm{a.data(), b.data(), sum.data(), norm.data(),
                                w ? static_cast<const float*>(w->data()) : nullptr, dt, a.element_count() / H, H, eps,
                                add_one ? 1 : 0};
        function_names_ = dt == PC_F32 ? "add_rmsnorm" : std::string("add_rmsnorm_") + dt_tag(dt);
    }
    const char* name() const override { return "AddRMSNorm"; }
    std::vector<Binding> tensors() const override {
        std::vector<Binding> v = {{a_, PC_ACCESS_READ}, {b_, PC_ACCESS_READ}, {sum_, PC_ACCESS_WRITE},
                                  {norm_, PC_ACCESS_WRITE}};
        if (has_w_) v.push_back({w_, PC_ACCESS_READ});
        return v;
    }
    void encode(KernelCommandEncoder& enc) const override {
        launch::AddRMSNorm p = p_;
        enc.dispatch(function_names_, tensors(), [p](cudaStream_t s) { return launch::add_rmsnorm(p, s); });
    }

private:
    Tensor a_, b_, sum_, norm_, w_;
    bool has_w_ = false;
    launch::AddRMSNorm p_{};
};

// ---------------------------------------------------------------------------
// Affine-quantized Matmul and embedding gathers (aq_matmul.cu)
// ---------------------------------------------------------------------------
// Checks of an AffineQuantizedTensor (AffineQuantizedTensor.swift:22-50) and
// the format subset the kernels serve (Matmul.swift:323-333).
void check_affine_quantized(const Tensor& packed, const Tensor& scales, const Tensor* biases, int64_t rows,
                            int64_t cols, int bits, int group, const char* what) {
    if (bits != 4 || group != 64)
        fail(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION,
             std::string(what) + " supports affine quantized tensors with bits=4, groupSize=64 only.");
    if (packed.dtype() != PC_U32)
        fail(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION,
             "AffineQuantizedTensor packed values must use u32 for packing uint32LittleEndian.");
    if (biases && (biases->dtype() != scales.dtype() || !biases->same_shape(scales)))
        fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "AffineQuantizedTensor scales and biases must share a data type and shape.");
    if (rows < 1 || cols < 1 || cols % group != 0)
        fail(PC_ERR_TENSOR_SHAPE_MISMATCH, std::string(what) + ": inner size " + std::to_string(cols) +
                                               " is not divisible by groupSize=" + std::to_string(group) + ".");
    require_elements(packed, rows * cols / 8, "packed values");
    require_elements(scales, rows * (cols / group), "scales");
    if (biases) require_elements(*biases, rows * (cols / group), "biases");
    if (!aligned16_ptr(packed.data()))
        fail(PC_ERR_TENSOR_SHAPE_MISMATCH, std::string(what) + ": packed values must be 16-byte aligned.");
}

class AqMatmulKernel : public Kernel {
public:
    AqMatmulKernel(Tensor a, Tensor packed, Tensor scales, const Tensor* biases, int64_t n, int64_t k, int bits,
                   int group, Tensor c)
        : a_(a), packed_(packed), scales_(scales), c_(c) {
        if (a.rank() != 2) fail(PC_ERR_TENSOR_INVALID_RANK, "expected rank 2, got rank " + std::to_string(a.rank()) + ".");
        if (c.rank() != 2) fail(PC_ERR_TENSOR_INVALID_RANK, "expected rank 2, got rank " + std::to_string(c.rank()) + ".");
        const int64_t m = a[0];
        if (a[1] != k)  // Matmul.swift:111-115
            fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "Matmul quantized RHS shape mismatch: a.shape=[" + std::to_string(m) +
                                                   "," + std::to_string(a[1]) + "] but b.inFeatures=" +
                                                   std::to_string(k) + ".");
        if (c[0] != m || c[1] != n)
            fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "Matmul output shape mismatch: expected [" + std::to_string(m) + "," +
                                                   std::to_string(n) + "], got " + c.shape_string() + ".");
        check_affine_quantized(packed, scales, biases, n, k, bits, group, "Matmul quantized RHS");
        const int xd = a.dtype(), sd = scales.dtype(), od = c.dtype();
        // Matmul.swift:323-333, plus the f16 extension
        const bool ok = (xd == PC_BF16 && sd == PC_BF16 && (od == PC_BF16 || od == PC_F32)) ||
                        (xd == PC_F32 && sd == PC_BF16 && od == PC_F32) ||
                        (xd == PC_F16 && sd == PC_F16 && od == PC_F16);
        if (!ok)
            fail(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION,
                 std::string("Unsupported affine quantized matmul combination: bits=4 groupSize=64, x=") +
                     dt_tag(xd) + ", scales=" + dt_tag(sd) + ", out=" + dt_tag(od) + ".");
        if (!aligned16_ptr(a.data()))
            fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "Matmul quantized: activations must be 16-byte aligned.");
        if (biases) {
            b_ = *biases;
            has_b_ = true;
        }
        p_ = launch::AqMatmul{a.data(), xd, static_cast<const uint32_t*>(packed.data()), scales.data(),
                              biases ? biases->data() : nullptr, sd, c.data(), od, m, n, k, 1, 0, 0, nullptr,
                              nullptr, nullptr};
        // Matmul.swift:302-304
        function_names_ = std::string(m == 1 ? "aq_qmv_fast_" : "aq_matvec_simd4_") + dt_tag(xd) + "_" + dt_tag(sd) +
                          "_" + dt_tag(od) + "_b4_g64";
    }
    const char* name() const override { return "Matmul"; }
    std::vector<Binding> tensors() const override {
        std::vector<Binding> v = {{a_, PC_ACCESS_READ}, {packed_, PC_ACCESS_READ}, {scales_, PC_ACCESS_READ},
                                  {c_, PC_ACCESS_WRITE}};
        if (has_b_) v.push_back({b_, PC_ACCESS_READ});
        return v;
    }
    void encode(KernelCommandEncoder& enc) const override {
        launch::AqMatmul p = p_;
        const int ks = enc.has_scratch() ? launch::aq_matmul_plan(p, enc.sm_count()) : 1;
        if (ks <= 1) {
            enc.dispatch(function_names_, tensors(), [p](cudaStream_t s) { return launch::aq_matmul(p, s); });
            return;
        }
        p.kslices = ks;
        std::vector<ScratchSpec> specs = {{{int64_t(launch::aq_matmul_workspace(p, ks))}, PC_U8}};
        enc.with_temporaries(specs, [&](const std::vector<Tensor>& t) {
            launch::AqMatmul q = p;
            q.workspace = t[0].data();
            std::vector<Binding> b = tensors();
            b.push_back({t[0], PC_ACCESS_READ_WRITE});
            enc.dispatch(function_names_, b, [q](cudaStream_t s) { return launch::aq_matmul(q, s); });
        });
    }

private:
    Tensor a_, packed_, scales_, c_, b_;
    bool has_b_ = false;
    launch::AqMatmul p_{};
};

// Fused decode forms of the quantized Matmul (TMA form only), each equal to
// a reference op sequence with its rounding points:
//   kNormMatmul: RMSNorm -> Matmul            (RMSNorm.metal, Matmul.swift:99-131)
//   kResidual:   Matmul -> Add(residual)      (Add.metal)
//   kGated:      RMSNorm -> Matmul [gate; up] (rows interleaved in 8s) -> act * up
//   kQKV:        RMSNorm -> Matmul [q; k; v] -> q, KVCacheWrite(k, v at pos)
struct AqWeight {
    Tensor packed, scales, biases;
    bool has_b = false;
    int64_t n = 0, k = 0;
    int bits = 0, group = 0;
};

AqWeight aq_weight_arg(const pc_affine_quantized* w, const char* what) {
    if (!w) fail(PC_ERR_TENSOR_SHAPE_MISMATCH, std::string(what) + " is null.");
    AqWeight r;
    r.packed = tensor_arg(w->packed, "packed");
    r.scales = tensor_arg(w->scales, "scales");
    if (w->biases) {
        r.biases = tensor_arg(w->biases, "biases");
        r.has_b = true;
    }
    r.n = w->out_features;
    r.k = w->in_features;
    r.bits = w->bits;
    r.group = w->group_size;
    check_affine_quantized(r.packed, r.scales, r.has_b ? &r.biases : nullptr, r.n, r.k, r.bits, r.group, what);
    return r;
}

class AqFusedKernel : public Kernel {
public:
    enum Form { kNormMatmul, kResidual, kGated, kQKV };
    AqFusedKernel(Form form, Tensor x, const Tensor* norm_w, float eps, bool add_one, const AqWeight& w, Tensor out,
                  const Tensor* residual, int activation, const Tensor* kc, const Tensor* vc, int64_t offset,
                  const Tensor* pos)
        : x_(x), w_(w), out_(out) {
        const int xd = x.dtype();
        if (!((xd == PC_BF16 && w.scales.dtype() == PC_BF16) || (xd == PC_F16 && w.scales.dtype() == PC_F16)))
            fail(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION, "fused 4-bit forms take bf16 x with bf16 scales, or f16 / f16.");
        if (out.dtype() != xd) fail(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION, "output dtype must be x's.");
        if (x.rank() != 2 || x[1] != w.k)
            fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "x must be [rows, " + std::to_string(w.k) + "]; got " + x.shape_string() + ".");
        if (!aligned16_ptr(x.data())) fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "x must be 16-byte aligned.");
        const int64_t m = x[0];
        launch::AqMatmul p{};
        p.x = x.data();
        p.x_dtype = xd;
        p.w = static_cast<const uint32_t*>(w.packed.data());
        p.scales = w.scales.data();
        p.biases = w.has_b ? w.biases.data() : nullptr;
        p.s_dtype = w.scales.dtype();
        p.out = out.data();
        p.out_dtype = xd;
        p.M = m;
        p.N = w.n;
        p.K = w.k;
        p.kslices = 1;
        if (form != kResidual) {
            p.norm = 1;
            p.eps = eps;
            p.add_one = add_one ? 1 : 0;
            if (norm_w) {
                if (norm_w->dtype() != PC_F32) fail(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION, "RMSNorm weight must be f32.");
                require_elements(*norm_w, w.k, "norm weight");
                p.norm_weight = static_cast<const float*>(norm_w->data());
                extra_.push_back({*norm_w, PC_ACCESS_READ});
            }
        }
        switch (form) {
        case kNormMatmul:
            p.epilogue = launch::kAqStore;
            if (out.rank() != 2 || out[0] != m || out[1] != w.n)
                fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "out must be [rows, out_features].");
            break;
        case kResidual:
            p.epilogue = launch::kAqResidual;
            if (out.rank() != 2 || out[0] != m || out[1] != w.n || !residual || !residual->same_shape(out) ||
                residual->dtype() != xd)
                fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "out and residual must be [rows, out_features] of x's dtype.");
            p.residual = residual->data();
            extra_.push_back({*residual, PC_ACCESS_READ});
            break;
        case kGated:
            p.epilogue = launch::kAqGated;
            if (activation != PC_ACT_GELU_TANH && activation != PC_ACT_SILU)
                fail(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION, "unknown activation.");
            p.activation = activation;
            if (w.n % 16 != 0 || out.rank() != 2 || out[0] != m || out[1] != w.n / 2)
                fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "gated: out_features = 2F with F % 8 == 0, out [rows, F].");
            break;
        case kQKV: {
            p.epilogue = launch::kAqQKV;
            if (!kc || !vc || kc->rank() != 4 || !kc->same_shape(*vc) || out.rank() != 4 || kc->dtype() != xd ||
                vc->dtype() != xd)
                fail(PC_ERR_TENSOR_INVALID_RANK, "QKV: q [B,Nq,1,Hd] and caches [B,Nkv,Smax,Hd] of x's dtype.");
            const int64_t B = out[0], Nq = out[1], Hd = out[3], Nkv = (*kc)[1], Smax = (*kc)[2];
            if (out[2] != 1 || B != m || (*kc)[0] != B || (*kc)[3] != Hd || (Nq + 2 * Nkv) * Hd != w.n)
                fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "QKV: out_features must be (Nq + 2 Nkv) * Hd, x [B, H].");
            if (!pos && (offset < 0 || offset >= Smax))
                fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "KV cache write offset " + std::to_string(offset) +
                                                       " outside cache length " + std::to_string(Smax) + ".");
            p.q_out = out.data();
            p.k_cache = kc->data();
            p.v_cache = vc->data();
            p.q_rows = Nq * Hd;
            p.kv_rows = Nkv * Hd;
            p.Hd = Hd;
            p.Smax = Smax;
            p.offset = offset;
            extra_.push_back({*kc, PC_ACCESS_WRITE});
            extra_.push_back({*vc, PC_ACCESS_WRITE});
            if (pos) {
                if (pos->dtype() != PC_I32 || pos->element_count() < 1)
                    fail(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION, "position must be int32 [1].");
                p.pos_dev = static_cast<const int32_t*>(pos->data());
                extra_.push_back({*pos, PC_ACCESS_READ});
            }
            break;
        }
        }
        launch::AqTmaPlan q{};
        if (!launch::aq_tma_plan(p, q))
            fail(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION,
                 "fused 4-bit forms need in_features % 256 == 0, 16-byte aligned packed values and 8-byte aligned "
                 "scales / biases.");
        p_ = p;
        function_names_ = std::string("aq_fused_") + dt_tag(xd) + "_b4_g64";
        name_ = form == kNormMatmul ? "AqRMSNormMatmul" : form == kResidual ? "AqMatmulResidual"
                : form == kGated ? "AqGatedMLP" : "AqQKVProjection";
    }
    const char* name() const override { return name_; }
    std::vector<Binding> tensors() const override {
        std::vector<Binding> v = {{x_, PC_ACCESS_READ}, {w_.packed, PC_ACCESS_READ}, {w_.scales, PC_ACCESS_READ},
                                  {out_, PC_ACCESS_WRITE}};
        if (w_.has_b) v.push_back({w_.biases, PC_ACCESS_READ});
        v.insert(v.end(), extra_.begin(), extra_.end());
        return v;
    }
    void encode(KernelCommandEncoder& enc) const override {
        launch::AqMatmul p = p_;
        enc.dispatch(function_names_, tensors(), [p](cudaStream_t s) { return launch::aq_matmul(p, s); });
    }

private:
    Tensor x_;
    AqWeight w_;
    Tensor out_;
    std::vector<Binding> extra_;
    launch::AqMatmul p_{};
    const char* name_ = "";
};

class EmbeddingGatherKernel : public Kernel {
public:
    // dense table: EmbeddingGather.swift:12-44
    EmbeddingGatherKernel(Tensor ids, Tensor table, Tensor out) : ids_(ids), table_(table), out_(out) {
        if (table.rank() != 2)
            fail(PC_ERR_TENSOR_INVALID_RANK, "expected rank 2, got rank " + std::to_string(table.rank()) + ".");
        if (out.rank() < 1 || ids.element_count() != out[0])
            fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "EmbeddingGather output first dimension must match ids element count; got " +
                                                   out.shape_string() + ", ids count " +
                                                   std::to_string(ids.element_count()) + ".");
        if (out.rank() != 2 || out[1] != table[1])
            fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "EmbeddingGather output shape must be [ids.count, " +
                                                   std::to_string(table[1]) + "]; got " + out.shape_string() + ".");
        if (ids.dtype() != PC_I32) fail(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION, "EmbeddingGather ids must be i32.");
        const int td = table.dtype(), od = out.dtype();
        const char* fn = nullptr;
        if (td == PC_F32 && od == PC_F32) fn = "embedding_gather";
        else if (td == PC_F16 && od == PC_F16) fn = "embedding_gather_f16";
        else if (td == PC_BF16 && od == PC_BF16) fn = "embedding_gather_bf16";
        else if (td == PC_BF16 && od == PC_F32) fn = "embedding_gather_bf16_to_f32";
        else
            fail(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION, std::string("Unsupported embedding gather data type combination: ") +
                                                               dt_tag(td) + ", " + dt_tag(od) + ".");
        function_names_ = fn;
        p_ = launch::EmbeddingGather{static_cast<const int32_t*>(ids.data()), table.data(), td, nullptr, nullptr,
                                     nullptr, out.data(), od, ids.element_count(), table[1], table[0]};
    }
    // quantized table: EmbeddingGather.swift:46-95
    EmbeddingGatherKernel(Tensor ids, Tensor packed, Tensor scales, const Tensor* biases, int64_t vocab, int64_t H,
                          int bits, int group, Tensor out)
        : ids_(ids), table_(packed), scales_(scales), out_(out), quantized_(true) {
        if (ids.rank() != 1)
            fail(PC_ERR_TENSOR_INVALID_RANK, "expected rank 1, got rank " + std::to_string(ids.rank()) + ".");
        if (ids.dtype() != PC_I32)
            fail(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION, "EmbeddingGather with quantized table requires i32 ids.");
        if (out.rank() != 2)
            fail(PC_ERR_TENSOR_INVALID_RANK, "expected rank 2, got rank " + std::to_string(out.rank()) + ".");
        if (out[0] != ids[0] || out[1] != H)
            fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "EmbeddingGather output shape mismatch: expected [" +
                                                   std::to_string(ids[0]) + "," + std::to_string(H) + "], got " +
                                                   out.shape_string() + ".");
        check_affine_quantized(packed, scales, biases, vocab, H, bits, group, "EmbeddingGather");
        const int sd = scales.dtype(), od = out.dtype();
        const bool ok = (sd == PC_BF16 && (od == PC_BF16 || od == PC_F32)) || (sd == PC_F16 && od == PC_F16);
        if (!ok)
            fail(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION, std::string("Unsupported quantized embedding gather: scales=") +
                                                               dt_tag(sd) + ", out=" + dt_tag(od) + ".");
        if (biases) {
            b_ = *biases;
            has_b_ = true;
        }
        function_names_ = std::string("aq_embedding_gather_") + dt_tag(sd) + "_" + dt_tag(od) + "_b4_g64";
        p_ = launch::EmbeddingGather{static_cast<const int32_t*>(ids.data()), nullptr, sd,
                                     static_cast<const uint32_t*>(packed.data()), scales.data(),
                                     biases ? biases->data() : nullptr, out.data(), od, ids[0], H, vocab};
    }
    const char* name() const override { return "EmbeddingGather"; }
    std::vector<Binding> tensors() const override {
        std::vector<Binding> v = {{ids_, PC_ACCESS_READ}, {table_, PC_ACCESS_READ}, {out_, PC_ACCESS_WRITE}};
        if (quantized_) v.push_back({scales_, PC_ACCESS_READ});
        if (has_b_) v.push_back({b_, PC_ACCESS_READ});
        return v;
    }
    void encode(KernelCommandEncoder& enc) const override {
        launch::EmbeddingGather p = p_;
        enc.dispatch(function_names_, tensors(), [p](cudaStream_t s) { return launch::embedding_gather(p, s); });
    }

private:
    Tensor ids_, table_, scales_, out_, b_;
    bool quantized_ = false, has_b_ = false;
    launch::EmbeddingGather p_{};
};

// ---------------------------------------------------------------------------
// Rotary embedding (rope.cu)
// ---------------------------------------------------------------------------
class RopeBuildCosSinKernel : public Kernel {
public:
    // RopeBuildCosSin.swift:31-50 (shape checks), :8-28 (constants)
    RopeBuildCosSinKernel(Tensor pos, Tensor inv, Tensor c, Tensor s, float scaling)
        : pos_(pos), inv_(inv), cos_(c), sin_(s), scaling_(scaling) {
        if (!c.same_shape(s))
            fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "RoPE cos and sin output shapes must match; got " + c.shape_string() +
                                                   " and " + s.shape_string() + ".");
        if (c.rank() != 2)
            fail(PC_ERR_TENSOR_INVALID_RANK, "expected rank 2, got rank " + std::to_string(c.rank()) + ".");
        T_ = c[0];
        Hd2_ = c[1];
        if (pos.element_count() != T_)
            fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "RoPE positions count must equal seqLen " + std::to_string(T_) +
                                                   "; got " + std::to_string(pos.element_count()) + ".");
        if (inv.element_count() != Hd2_)
            fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "RoPE invFreq count must equal halfHeadDim " + std::to_string(Hd2_) +
                                                   "; got " + std::to_string(inv.element_count()) + ".");
        if (pos.dtype() != PC_I32 || inv.dtype() != PC_F32 || c.dtype() != PC_F32 || s.dtype() != PC_F32)
            fail(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION, "RoPE tables: int32 positions, f32 invFreq and tables.");
        function_names_ = "rope_build_cos_sin";
    }
    const char* name() const override { return "RopeBuildCosSin"; }
    std::vector<Binding> tensors() const override {
        return {{pos_, PC_ACCESS_READ}, {inv_, PC_ACCESS_READ}, {cos_, PC_ACCESS_WRITE}, {sin_, PC_ACCESS_WRITE}};
    }
    void encode(KernelCommandEncoder& enc) const override {
        const int32_t* pos = static_cast<const int32_t*>(pos_.data());
        const float* inv = static_cast<const float*>(inv_.data());
        float* c = static_cast<float*>(cos_.data());
        float* sn = static_cast<float*>(sin_.data());
        const int64_t T = T_, Hd2 = Hd2_;
        const float sc = scaling_;
        enc.dispatch(function_names_, tensors(),
                     [=](cudaStream_t s) { return launch::rope_build_cos_sin(pos, inv, c, sn, T, Hd2, sc, s); });
    }

private:
    Tensor pos_, inv_, cos_, sin_;
    float scaling_;
    int64_t T_ = 0, Hd2_ = 0;
};

class RopeApplyKernel : public Kernel {
public:
    // RopeApply.swift:48-64 (shape checks), :19-31 (dtype routing)
    RopeApplyKernel(Tensor x, Tensor c, Tensor s, Tensor out) : x_(x), cos_(c), sin_(s), out_(out) {
        if (x.rank() != 4)
            fail(PC_ERR_TENSOR_INVALID_RANK, "expected rank 4, got rank " + std::to_string(x.rank()) + ".");
        if (!x.same_shape(out))
            fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "RoPE output shape must match input; got " + out.shape_string() +
                                                   ", expected " + x.shape_string() + ".");
        const int64_t Hd = x[3];
        if (Hd % 2 != 0)
            fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "RoPE head dimension must be even; got " + std::to_string(Hd) + ".");
        if (c.rank() != 2 || s.rank() != 2 || c[0] != x[1] || c[1] != Hd / 2 || !c.same_shape(s))
            fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "RoPE tables must have shape [" + std::to_string(x[1]) + ", " +
                                                   std::to_string(Hd / 2) + "]; got cos " + c.shape_string() +
                                                   ", sin " + s.shape_string() + ".");
        const int xd = x.dtype(), td = c.dtype();
        const bool ok = s.dtype() == td && out.dtype() == xd &&
                        ((xd == PC_F32 && td == PC_F32) || (xd == PC_BF16 && (td == PC_BF16 || td == PC_F32)) ||
                         (xd == PC_F16 && (td == PC_F16 || td == PC_F32)));
        if (!ok)
            fail(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION, std::string("Unsupported RoPE data type combination: ") +
                                                               dt_tag(xd) + ", " + dt_tag(td) + ".");
        p_ = launch::RopeApply{x.data(), c.data(), s.data(), out.data(), xd, td, xd, x[0], x[1], x[2], Hd / 2};
        if (xd == PC_F32) function_names_ = "rope_apply";
        else if (td == PC_F32) function_names_ = std::string("rope_apply_f32_tables_") + dt_tag(xd);
        else function_names_ = std::string("rope_apply_") + dt_tag(xd);
    }
    const char* name() const override { return "RopeApply"; }
    std::vector<Binding> tensors() const override {
        return {{x_, PC_ACCESS_READ}, {cos_, PC_ACCESS_READ}, {sin_, PC_ACCESS_READ}, {out_, PC_ACCESS_WRITE}};
    }
    void encode(KernelCommandEncoder& enc) const override {
        launch::RopeApply p = p_;
        enc.dispatch(function_names_, tensors(), [p](cudaStream_t s) { return launch::rope_apply(p, s); });
    }

private:
    Tensor x_, cos_, sin_, out_;
    launch::RopeApply p_{};
};

// The decode step's RMSNorm(q) -> RopeApply, RMSNorm(k) -> RopeApply,
// RMSNorm(v) (Gemma4TextInference.swift:352-381) in place, one launch.
class QKNormRopeKernel : public Kernel {
public:
    QKNormRopeKernel(Tensor q, Tensor kc, Tensor vc, Tensor qn, Tensor kn, Tensor c, Tensor s, float eps,
                     bool add_one, bool norm_v, int64_t offset, const Tensor* pos)
        : q_(q), kc_(kc), vc_(vc), qn_(qn), kn_(kn), cos_(c), sin_(s) {
        const int dt = q.dtype();
        if (!is_float(dt) || kc.dtype() != dt || vc.dtype() != dt)
            fail(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION, "QKNormRope needs one float dtype for q and the caches.");
        if (qn.dtype() != PC_F32 || kn.dtype() != PC_F32 || c.dtype() != PC_F32 || s.dtype() != PC_F32)
            fail(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION, "QKNormRope norm weights and tables must be f32.");
        if (q.rank() != 4 || kc.rank() != 4 || !kc.same_shape(vc) || c.rank() != 2 || !c.same_shape(s))
            fail(PC_ERR_TENSOR_INVALID_RANK, "QKNormRope wants q [B,Nq,1,Hd], caches [B,Nkv,Smax,Hd], tables [R,Hd/2].");
        const int64_t B = q[0], Nq = q[1], Hd = q[3], Nkv = kc[1], Smax = kc[2];
        if (q[2] != 1 || kc[0] != B || kc[3] != Hd || c[1] != Hd / 2)
            fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "QKNormRope shapes disagree: q " + q.shape_string() + ", cache " +
                                                   kc.shape_string() + ", table " + c.shape_string() + ".");
        if (Hd % 2 != 0 || Hd > 2048)
            fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "QKNormRope head dimension must be even and <= 2048.");
        require_elements(qn, Hd, "q norm weight");
        require_elements(kn, Hd, "k norm weight");
        if (!pos && (offset < 0 || offset >= Smax || (c[0] != 1 && offset >= c[0])))
            fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "QKNormRope position " + std::to_string(offset) +
                                                   " outside the cache or the tables.");
        if (pos) {
            if (pos->dtype() != PC_I32 || pos->element_count() < 1)
                fail(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION, "position must be int32 [1].");
            pos_ = *pos;
            has_pos_ = true;
        }
        p_ = launch::QKNormRope{q.data(), kc.data(), vc.data(), static_cast<const float*>(qn.data()),
                                static_cast<const float*>(kn.data()), static_cast<const float*>(c.data()),
                                static_cast<const float*>(s.data()), dt, B, Nq, Nkv, Hd, Smax, offset, c[0],
                                pos ? static_cast<const int32_t*>(pos->data()) : nullptr, eps, add_one ? 1 : 0,
                                norm_v ? 1 : 0};
        function_names_ = dt == PC_F32 ? "qk_norm_rope" : std::string("qk_norm_rope_") + dt_tag(dt);
    }
    const char* name() const override { return "QKNormRope"; }
    std::vector<Binding> tensors() const override {
        std::vector<Binding> b = {{q_, PC_ACCESS_READ_WRITE}, {kc_, PC_ACCESS_READ_WRITE}, {vc_, PC_ACCESS_READ_WRITE},
                                  {qn_, PC_ACCESS_READ},       {kn_, PC_ACCESS_READ},        {cos_, PC_ACCESS_READ},
                                  {sin_, PC_ACCESS_READ}};
        if (has_pos_) b.push_back({pos_, PC_ACCESS_READ});
        return b;
    }
    void encode(KernelCommandEncoder& enc) const override {
        launch::QKNormRope p = p_;
        enc.dispatch(function_names_, tensors(), [p](cudaStream_t s) { return launch::qk_norm_rope(p, s); });
    }

private:
    Tensor q_, kc_, vc_, qn_, kn_, cos_, sin_, pos_;
    bool has_pos_ = false;
    launch::QKNormRope p_{};
};

// ---------------------------------------------------------------------------
// All-reduce + Add + RMSNorm over peer memory (allreduce.cu)
// ---------------------------------------------------------------------------
class PeerAllReduceKernel : public Kernel {
public:
    PeerAllReduceKernel(const pc_peer_group* g, int buffer, Tensor res, const Tensor* w, float eps, bool add_one,
                        Tensor sum, Tensor norm)
        : res_(res), sum_(sum), norm_(norm) {
        if (!g) fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "peer group is null.");
        const int dt = res.dtype();
        if ((dt != PC_BF16 && dt != PC_F16) || sum.dtype() != dt || norm.dtype() != dt)
            fail(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION, "peer all-reduce serves bf16 or f16.");
        if (!res.same_shape(sum) || !res.same_shape(norm) || res.rank() < 1)
            fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "residual, sum and norm outputs must have one shape.");
        if (g->world < 1 || g->world > PC_MAX_PEERS || g->rank < 0 || g->rank >= g->world)
            fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "peer group: bad world / rank.");
        launch::PeerAllReduce p{};
        for (int r = 0; r < g->world; ++r) {
            if (!g->partial[r][0] || !g->partial[r][1] || !g->control[r])
                fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "peer group: missing buffer of rank " + std::to_string(r) + ".");
            p.partial[r][0] = g->partial[r][0];
            p.partial[r][1] = g->partial[r][1];
            p.ctl[r] = g->control[r];
        }
        const int64_t H = res[res.rank() - 1];
        if (w) {
            if (w->dtype() != PC_F32) fail(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION, "RMSNorm weight must be f32.");
            require_elements(*w, H, "all-reduce norm weight");
            w_ = *w;
            has_w_ = true;
        }
        p.rank = g->rank;
        p.world = g->world;
        p.buffer = buffer;
        p.residual = res.data();
        p.sum_out = sum.data();
        p.norm_out = norm.data();
        p.weight = w ? static_cast<const float*>(w->data()) : nullptr;
        p.dtype = dt;
        p.rows = res.element_count() / H;
        p.H = H;
        p.eps = eps;
        p.add_one = add_one ? 1 : 0;
        if (!launch::peer_allreduce_supports(p))
            fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "peer all-reduce: H must be a multiple of 8 and <= 8192, buffer 0 or 1.");
        p_ = p;
        function_names_ = dt == PC_BF16 ? "allreduce_add_rmsnorm_bf16" : "allreduce_add_rmsnorm_f16";
    }
    const char* name() const override { return "AllReduceAddRMSNorm"; }
    std::vector<Binding> tensors() const override {
        std::vector<Binding> v = {{res_, PC_ACCESS_READ}, {sum_, PC_ACCESS_WRITE}, {norm_, PC_ACCESS_WRITE}};
        if (has_w_) v.push_back({w_, PC_ACCESS_READ});
        return v;
    }
    void encode(KernelCommandEncoder& enc) const override {
        launch::PeerAllReduce p = p_;
        enc.dispatch(function_names_, tensors(), [p](cudaStream_t s) { return launch::peer_allreduce_add_rmsnorm(p, s); });
    }

private:
    Tensor res_, sum_, norm_, w_;
    bool has_w_ = false;
    launch::PeerAllReduce p_{};
};

// The peer all-reduce parameters from a group descriptor (validated).
launch::PeerAllReduce peer_params(const pc_peer_group* g, int buffer, const Tensor& res, const Tensor* w, float eps,
                                  bool add_one, const Tensor& sum, const Tensor& norm) {
    if (!g) fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "peer group is null.");
    const int dt = res.dtype();
    if ((dt != PC_BF16 && dt != PC_F16) || sum.dtype() != dt || norm.dtype() != dt)
        fail(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION, "peer all-reduce serves bf16 or f16.");
    if (!res.same_shape(sum) || !res.same_shape(norm) || res.rank() < 1)
        fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "residual, sum and norm outputs must have one shape.");
    if (g->world < 1 || g->world > PC_MAX_PEERS || g->rank < 0 || g->rank >= g->world)
        fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "peer group: bad world / rank.");
    launch::PeerAllReduce p{};
    for (int r = 0; r < g->world; ++r) {
        if (!g->partial[r][0] || !g->partial[r][1] || !g->control[r])
            fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "peer group: missing buffer of rank " + std::to_string(r) + ".");
        p.partial[r][0] = g->partial[r][0];
        p.partial[r][1] = g->partial[r][1];
        p.ctl[r] = g->control[r];
    }
    const int64_t H = res[res.rank() - 1];
    if (w) {
        if (w->dtype() != PC_F32) fail(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION, "RMSNorm weight must be f32.");
        require_elements(*w, H, "all-reduce norm weight");
    }
    p.rank = g->rank;
    p.world = g->world;
    p.buffer = buffer;
    p.residual = res.data();
    p.sum_out = sum.data();
    p.norm_out = norm.data();
    p.weight = w ? static_cast<const float*>(w->data()) : nullptr;
    p.dtype = dt;
    p.rows = res.element_count() / H;
    p.H = H;
    p.eps = eps;
    p.add_one = add_one ? 1 : 0;
    if (!launch::peer_allreduce_supports(p))
        fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "peer all-reduce: H must be a multiple of 8 and <= 8192, buffer 0 or 1.");
    return p;
}

class MatmulAllReduceKernel : public Kernel {
public:
    MatmulAllReduceKernel(Tensor a, Tensor w, const pc_peer_group* g, int buffer, Tensor res, const Tensor* nw,
                          float eps, bool add_one, Tensor sum, Tensor norm)
        : a_(a), w_(w), res_(res), sum_(sum), norm_(norm) {
        ar_ = peer_params(g, buffer, res, nw, eps, add_one, sum, norm);
        if (nw) {
            nw_ = *nw;
            has_nw_ = true;
        }
        if (a.rank() != 2 || w.rank() != 2 || a[1] != w[1] || ar_.rows != a[0] || ar_.H != w[0])
            fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "MatmulAllReduce wants a [M,K], w [N,K], residual [M,N]; got a " +
                                                   a.shape_string() + ", w " + w.shape_string() + ".");
        if (a.dtype() != res.dtype() || w.dtype() != a.dtype())
            fail(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION, "MatmulAllReduce needs one 16-bit dtype.");
        mm_ = launch::Matmul{a.data(), a.dtype(), w.data(), w.dtype(), const_cast<void*>(ar_.partial[ar_.rank][buffer]),
                             a.dtype(), a[0], a[1], w[0], 1};
        if (!launch::tcgen05_supports_skinny(mm_))
            fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "MatmulAllReduce serves the tensor-core GEMM with M <= 64, K % 8 == 0.");
        function_names_ = "matmul_tc_bf16_tb";
    }
    const char* name() const override { return "MatmulAllReduceAddRMSNorm"; }
    std::vector<Binding> tensors() const override {
        std::vector<Binding> v = {{a_, PC_ACCESS_READ}, {w_, PC_ACCESS_READ}, {res_, PC_ACCESS_READ},
                                  {sum_, PC_ACCESS_WRITE}, {norm_, PC_ACCESS_WRITE}};
        if (has_nw_) v.push_back({nw_, PC_ACCESS_READ});
        return v;
    }
    void encode(KernelCommandEncoder& enc) const override {
        launch::Matmul p = mm_;
        launch::PeerAllReduce ar = ar_;
        const size_t ws = enc.has_scratch() ? launch::matmul_tcgen05_workspace(p) : 0;
        if (ws == 0) {
            enc.dispatch(function_names_, tensors(),
                         [p, ar](cudaStream_t s) { return launch::matmul_tcgen05_allreduce(p, ar, s); });
            return;
        }
        std::vector<ScratchSpec> specs = {{{int64_t(ws)}, PC_U8}};
        enc.with_temporaries(specs, [&](const std::vector<Tensor>& t) {
            launch::Matmul q = p;
            q.workspace = t[0].data();
            std::vector<Binding> b = tensors();
            b.push_back({t[0], PC_ACCESS_READ_WRITE});
            enc.dispatch(function_names_, b, [q, ar](cudaStream_t s) { return launch::matmul_tcgen05_allreduce(q, ar, s); });
        });
    }

private:
    Tensor a_, w_, res_, sum_, norm_, nw_;
    bool has_nw_ = false;
    launch::Matmul mm_{};
    launch::PeerAllReduce ar_{};
};

// ---------------------------------------------------------------------------
// Fused decode step (decode_step.cu)
// ---------------------------------------------------------------------------
launch::DecodeStep make_step(const pc_decode_stack_desc* d) {
    if (!d) fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "descriptor is null.");
    if (d->dtype != PC_F16 && d->dtype != PC_BF16)
        fail(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION, "decode stack needs f16 or bf16.");
    if (d->num_layers < 1 || d->hidden < 8 || d->ffn < 8 || d->max_ctx < 1 || d->q_heads < 1 || d->kv_heads < 1)
        fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "decode stack dimensions must be positive.");
    if (d->q_heads % d->kv_heads != 0)
        fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "query heads must be divisible by KV heads.");
    if (d->activation != PC_ACT_GELU_TANH && d->activation != PC_ACT_SILU)
        fail(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION, "unknown activation.");
    if (!d->layers || !d->x || !d->x2 || !d->h || !d->q || !d->attn || !d->act || !d->position)
        fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "decode stack buffers must all be given.");
    launch::DecodeStep p{};
    p.layers = reinterpret_cast<const launch::DecodeLayer*>(d->layers);
    p.L = d->num_layers;
    p.H = d->hidden; p.Nq = d->q_heads; p.Nkv = d->kv_heads; p.Hd = d->head_dim; p.F = d->ffn; p.Smax = d->max_ctx;
    p.eps = d->eps; p.scale = d->attn_scale; p.activation = d->activation; p.add_one = d->add_one_to_weight != 0;
    p.dtype = d->dtype;
    p.x = d->x; p.x2 = d->x2; p.h = d->h; p.q = d->q; p.attn = d->attn; p.act = d->act; p.pos = d->position;
    static_assert(sizeof(pc_decode_layer) == sizeof(launch::DecodeLayer), "decode layer table layout");
    p.qk_norm = d->qk_norm != 0;
    p.norm_v = d->norm_v != 0;
    if (d->rope_rows < 0) fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "rope_rows must be >= 0.");
    p.has_rope = d->rope_rows > 0;
    p.rope_rows = d->rope_rows < 1 ? 1 : d->rope_rows;
    int dev = 0;
    cudaGetDevice(&dev);
    p.grid = launch::device_info(dev).sm_count;
    if (!launch::decode_step_plan(p, p.grid))
        fail(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION,
             "fused decode step serves head dim 256, Nq/Nkv in {1,2,4}, hidden/ffn multiples of 8.");
    return p;
}

class DecodeStackKernel : public Kernel {
public:
    explicit DecodeStackKernel(const pc_decode_stack_desc* d) : p_(make_step(d)) {
        const size_t need = launch::decode_step_workspace_bytes(p_);
        if (!d->workspace || d->workspace_bytes < need)
            fail(PC_ERR_WORKSPACE_EXHAUSTED, "decode stack workspace needs " + std::to_string(need) + " bytes; got " +
                                                 std::to_string(d->workspace_bytes) + ".");
        char* ws = static_cast<char*>(d->workspace);
        const size_t o = size_t(p_.Nq) * p_.splits * p_.Hd * 4, ml = size_t(p_.Nq) * p_.splits * 4;
        p_.counters = reinterpret_cast<unsigned int*>(ws);
        size_t off = (size_t(p_.L * 6 + 1 + p_.L * p_.Nkv) * 4 + 255) / 256 * 256;
        p_.po = reinterpret_cast<float*>(ws + off);
        p_.pm = reinterpret_cast<float*>(ws + off + o);
        p_.pl = reinterpret_cast<float*>(ws + off + o + ml);
        function_names_ = std::string(p_.qk_norm || p_.has_rope ? "decode_step_qk_" : "decode_step_") +
                          (d->dtype == PC_BF16 ? "bf16" : "f16");
        auto t = [](void* ptr, int64_t n, int dt) {
            pc_tensor x{};
            x.data = ptr;
            x.dtype = dt;
            x.rank = 1;
            x.shape[0] = n;
            return Tensor(x);
        };
        int dt = d->dtype;
        bindings_ = {{t(d->x, p_.H, dt), PC_ACCESS_READ_WRITE}, {t(d->x2, p_.H, dt), PC_ACCESS_READ_WRITE},
                     {t(d->h, p_.H, dt), PC_ACCESS_READ_WRITE}, {t(d->q, p_.Nq * p_.Hd, dt), PC_ACCESS_READ_WRITE},
                     {t(d->attn, p_.Nq * p_.Hd, dt), PC_ACCESS_READ_WRITE}, {t(d->act, p_.F, dt), PC_ACCESS_READ_WRITE},
                     {t(d->workspace, int64_t(need), PC_U8), PC_ACCESS_READ_WRITE},
                     {t(const_cast<int32_t*>(d->position), 1, PC_I32), PC_ACCESS_READ}};
    }
    const char* name() const override { return "DecodeStack"; }
    std::vector<Binding> tensors() const override { return bindings_; }
    void encode(KernelCommandEncoder& enc) const override {
        launch::DecodeStep p = p_;
        enc.dispatch(function_names_, bindings_, [p](cudaStream_t s) { return launch::decode_step(p, s); });
    }

private:
    launch::DecodeStep p_;
    std::vector<Binding> bindings_;
};

}  // namespace
}  // namespace popcorn

using namespace popcorn;

struct pc_kernel {
    std::unique_ptr<Kernel> impl;
    std::vector<Binding> bindings;
};

namespace {
int wrap(std::unique_ptr<Kernel> k, pc_kernel** out) {
    auto* pk = new pc_kernel{std::move(k), {}};
    pk->bindings = pk->impl->tensors();
    *out = pk;
    return PC_OK;
}
}  // namespace

#define PC_GUARD_BEGIN                       \
    try {                                    \
        if (kernel) *kernel = nullptr;
#define PC_GUARD_END                         \
    }                                        \
    catch (const PopcornError& e) {          \
        set_last_error(e.message);           \
        return e.code;                       \
    }                                        \
    catch (const std::exception& e) {        \
        set_last_error(e.what());            \
        return PC_ERR_GPU_INTERNAL;          \
    }

extern "C" {

void pc_kernel_destroy(pc_kernel* kernel) { delete kernel; }

const char* pc_kernel_name(const pc_kernel* kernel) { return kernel ? kernel->impl->name() : ""; }

int pc_kernel_binding_count(const pc_kernel* kernel) { return kernel ? int(kernel->bindings.size()) : 0; }

int pc_kernel_binding(const pc_kernel* kernel, int index, pc_tensor* tensor, int* access) {
    if (!kernel || index < 0 || size_t(index) >= kernel->bindings.size()) {
        set_last_error("binding index out of range.");
        return PC_ERR_TENSOR_SHAPE_MISMATCH;
    }
    if (tensor) *tensor = kernel->bindings[size_t(index)].tensor.d;
    if (access) *access = kernel->bindings[size_t(index)].access;
    return PC_OK;
}

int pc_kernel_set_l2_prefetch(pc_kernel* kernel, int32_t slot, const void* ptr, uint64_t bytes) {
    try {
        if (!kernel) fail(PC_ERR_KERNEL_FUNCTION_NOT_FOUND, "kernel is null.");
        kernel->impl->set_prefetch(slot, ptr, bytes);
    } catch (const PopcornError& e) {
        set_last_error(e.message);
        return e.code;
    }
    return PC_OK;
}

int pc_kernel_set_hint(pc_kernel* kernel, int32_t hint, int64_t value) {
    try {
        if (!kernel) fail(PC_ERR_KERNEL_FUNCTION_NOT_FOUND, "kernel is null.");
        kernel->impl->set_hint(hint, value);
    } catch (const PopcornError& e) {
        set_last_error(e.message);
        return e.code;
    }
    return PC_OK;
}

const char* pc_kernel_function_names(const pc_kernel* kernel) {
    return kernel ? kernel->impl->function_names().c_str() : "";
}

// FlashAttention.route, FlashAttention.swift:109-113. Sq == 1 -> decoding;
// Sq >= 32 with a 16-bit dtype and hd in the tensor-core kernel's set ->
// tensor; otherwise plain. (The final decision for "tensor" also checks
// shapes in the launcher; pc_kernel_function_names shows the result.)
int pc_flash_attention_route(int64_t query_len, int64_t head_dim, int32_t dtype) {
    if (query_len == 1) return PC_PATH_DECODING;
    if (query_len >= 32 && head_dim <= 512 && (dtype == PC_BF16 || dtype == PC_F16)) return PC_PATH_TENSOR;
    return PC_PATH_PLAIN;
}

int pc_encoder_encode(pc_encoder* encoder, const pc_kernel* k) {
    try {
        if (!encoder || !k) fail(PC_ERR_KERNEL_FUNCTION_NOT_FOUND, "encoder or kernel is null.");
        encoder_impl(encoder).encode(*k->impl);
    } catch (const PopcornError& e) {
        set_last_error(e.message);
        return e.code;
    } catch (const std::exception& e) {
        set_last_error(e.what());
        return PC_ERR_GPU_INTERNAL;
    }
    return PC_OK;
}

int pc_kernel_flash_attention_dims(const pc_tensor* q, const pc_tensor* k, const pc_tensor* v, const pc_tensor* out,
                                   int64_t batch, int64_t query_heads, int64_t kv_heads, int64_t query_len,
                                   int64_t key_len, int64_t head_dim, float scale, pc_attention_mask mask,
                                   pc_kernel** kernel) {
    PC_GUARD_BEGIN
    return wrap(std::make_unique<FlashAttentionKernel>(tensor_arg(q, "q"), tensor_arg(k, "k"), tensor_arg(v, "v"),
                                                       tensor_arg(out, "out"), nullptr, batch, query_heads, kv_heads,
                                                       query_len, key_len, head_dim, scale, mask),
                kernel);
    PC_GUARD_END
}

// FlashAttention.swift:51-90.
int pc_kernel_flash_attention(const pc_tensor* q, const pc_tensor* k, const pc_tensor* v, const pc_tensor* out,
                              float scale, pc_attention_mask mask, pc_kernel** kernel) {
    PC_GUARD_BEGIN
    Tensor tq = tensor_arg(q, "q"), tk = tensor_arg(k, "k"), tv = tensor_arg(v, "v"), to = tensor_arg(out, "out");
    require_rank(tq, 4);
    require_rank(tk, 4);
    require_rank(tv, 4);
    int64_t B = tq[0], Nq = tq[1], Sq = tq[2], Hd = tq[3], Nkv = tk[1], Sk = tk[2];
    if (tk[0] != B || tk[3] != Hd)
        fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "FlashAttention K shape must match Q batch/headDim; q " + tq.shape_string() +
                                               ", k " + tk.shape_string() + ".");
    if (!tv.same_shape(tk))
        fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "FlashAttention V shape must match K; v " + tv.shape_string() + ", k " +
                                               tk.shape_string() + ".");
    std::vector<int64_t> expected = {B, Nq, Sq, Hd};
    if (to.dims() != expected)
        fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "FlashAttention output shape must be " + dims_string(expected) + "; got " +
                                               to.shape_string() + ".");
    return wrap(std::make_unique<FlashAttentionKernel>(tq, tk, tv, to, nullptr, B, Nq, Nkv, Sq, Sk, Hd, scale, mask),
                kernel);
    PC_GUARD_END
}

int pc_kernel_flash_decoding_ragged(const pc_tensor* q, const pc_tensor* k_cache, const pc_tensor* v_cache,
                                    const pc_tensor* seq_lens, const pc_tensor* out, float scale,
                                    pc_attention_mask mask, pc_kernel** kernel) {
    PC_GUARD_BEGIN
    Tensor tq = tensor_arg(q, "q"), tk = tensor_arg(k_cache, "k_cache"), tv = tensor_arg(v_cache, "v_cache"),
           tl = tensor_arg(seq_lens, "seq_lens"), to = tensor_arg(out, "out");
    require_rank(tq, 4);
    require_rank(tk, 4);
    int64_t B = tq[0], Nq = tq[1], Sq = tq[2], Hd = tq[3], Nkv = tk[1], Smax = tk[2];
    if (Sq != 1) fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "ragged FlashDecoding takes one query token per sequence.");
    if (tk[0] != B || tk[3] != Hd || !tv.same_shape(tk))
        fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "K/V caches must be [B,Nkv,Smax,Hd] matching q; q " + tq.shape_string() +
                                               ", k " + tk.shape_string() + ", v " + tv.shape_string() + ".");
    if (to.dims() != tq.dims())
        fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "FlashDecoding output shape must be " + tq.shape_string() + "; got " +
                                               to.shape_string() + ".");
    if (Smax < 1) fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "KV cache length must be >= 1.");
    return wrap(std::make_unique<FlashAttentionKernel>(tq, tk, tv, to, &tl, B, Nq, Nkv, 1, Smax, Hd, scale, mask), kernel);
    PC_GUARD_END
}

int pc_kernel_kv_cache_write_dims(const pc_tensor* source, const pc_tensor* cache, int64_t batch, int64_t kv_heads,
                                  int64_t new_len, int64_t max_len, int64_t head_dim, int64_t offset,
                                  pc_kernel** kernel) {
    PC_GUARD_BEGIN
    return wrap(std::make_unique<KVCacheWriteKernel>(tensor_arg(source, "source"), tensor_arg(cache, "cache"), batch,
                                                     kv_heads, new_len, max_len, head_dim, offset),
                kernel);
    PC_GUARD_END
}

// KVCacheWrite.swift:38-49.
int pc_kernel_kv_cache_write(const pc_tensor* source, const pc_tensor* cache, int64_t offset, pc_kernel** kernel) {
    PC_GUARD_BEGIN
    Tensor s = tensor_arg(source, "source"), c = tensor_arg(cache, "cache");
    require_rank(s, 4);
    require_rank(c, 4);
    if (c[0] != s[0] || c[1] != s[1] || c[3] != s[3])
        fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "KV cache shape must match source batch/heads/headDim; source " +
                                               s.shape_string() + ", cache " + c.shape_string() + ".");
    return wrap(std::make_unique<KVCacheWriteKernel>(s, c, s[0], s[1], s[2], c[2], s[3], offset), kernel);
    PC_GUARD_END
}

int pc_kernel_rmsnorm_dims(const pc_tensor* x, const pc_tensor* weight, const pc_tensor* out, int64_t row_count,
                           int64_t hidden_size, float eps, int32_t add_one_to_weight, pc_kernel** kernel) {
    PC_GUARD_BEGIN
    Tensor w;
    if (weight) w = tensor_arg(weight, "weight");
    return wrap(std::make_unique<RMSNormKernel>(tensor_arg(x, "x"), weight ? &w : nullptr, tensor_arg(out, "out"),
                                                row_count, hidden_size, eps, add_one_to_weight != 0),
                kernel);
    PC_GUARD_END
}

// RMSNorm.swift:39-70.
int pc_kernel_rmsnorm(const pc_tensor* x, const pc_tensor* weight, const pc_tensor* out, int32_t axis, float eps,
                      int32_t add_one_to_weight, pc_kernel** kernel) {
    PC_GUARD_BEGIN
    Tensor tx = tensor_arg(x, "x"), to = tensor_arg(out, "out");
    int rank = tx.rank();
    int norm_axis = axis < 0 ? rank + axis : axis;
    if (rank <= 0 || norm_axis != rank - 1)
        fail(PC_ERR_TENSOR_INVALID_AXIS, "Axis " + std::to_string(axis) + " is invalid for a tensor of rank " +
                                             std::to_string(rank) + ".");
    if (!tx.same_shape(to))
        fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "RMSNorm output shape must match input; got " + to.shape_string() +
                                               ", expected " + tx.shape_string() + ".");
    int64_t H = tx[norm_axis];
    int64_t rows = H > 0 ? tx.element_count() / H : 0;
    Tensor w;
    if (weight) {
        w = tensor_arg(weight, "weight");
        bool ok = (w.rank() == 1 && w[0] == H) || w.same_shape(tx);
        if (!ok)
            fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "RMSNorm weight shape must be [" + std::to_string(H) + "] or " +
                                                   tx.shape_string() + "; got " + w.shape_string() + ".");
    }
    return wrap(std::make_unique<RMSNormKernel>(tx, weight ? &w : nullptr, to, rows, H, eps, add_one_to_weight != 0),
                kernel);
    PC_GUARD_END
}

int pc_kernel_matmul_dims(const pc_tensor* a, const pc_tensor* b, const pc_tensor* c, int64_t m, int64_t k, int64_t n,
                          int32_t transpose_b, pc_kernel** kernel) {
    PC_GUARD_BEGIN
    return wrap(std::make_unique<MatmulKernel>(tensor_arg(a, "a"), tensor_arg(b, "b"), tensor_arg(c, "c"), m, k, n,
                                               transpose_b != 0),
                kernel);
    PC_GUARD_END
}

// Matmul.swift:68-93.
int pc_kernel_matmul(const pc_tensor* a, const pc_tensor* b, const pc_tensor* c, int32_t transpose_b, pc_kernel** kernel) {
    PC_GUARD_BEGIN
    Tensor ta = tensor_arg(a, "a"), tb = tensor_arg(b, "b"), tc = tensor_arg(c, "c");
    require_rank(ta, 2);
    require_rank(tb, 2);
    require_rank(tc, 2);
    int64_t m = ta[0], k = ta[1];
    int64_t n = transpose_b ? tb[0] : tb[1];
    std::vector<int64_t> eb = transpose_b ? std::vector<int64_t>{n, k} : std::vector<int64_t>{k, n};
    std::vector<int64_t> ec = {m, n};
    if (tb.dims() != eb)
        fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "Matmul RHS shape mismatch: expected " + dims_string(eb) + ", got " +
                                               tb.shape_string() + ".");
    if (tc.dims() != ec)
        fail(PC_ERR_TENSOR_SHAPE_MISMATCH, "Matmul output shape mismatch: expected " + dims_string(ec) + ", got " +
                                               tc.shape_string() + ".");
    return wrap(std::make_unique<MatmulKernel>(ta, tb, tc, m, k, n, transpose_b != 0), kernel);
    PC_GUARD_END
}

int pc_kernel_gelu_tanh(const pc_tensor* x, const pc_tensor* out, pc_kernel** kernel) {
    PC_GUARD_BEGIN
    return wrap(std::make_unique<UnaryKernel>(launch::Unary::kGeluTanh, tensor_arg(x, "x"), tensor_arg(out, "out")), kernel);
    PC_GUARD_END
}

int pc_kernel_silu(const pc_tensor* x, const pc_tensor* out, pc_kernel** kernel) {
    PC_GUARD_BEGIN
    return wrap(std::make_unique<UnaryKernel>(launch::Unary::kSilu, tensor_arg(x, "x"), tensor_arg(out, "out")), kernel);
    PC_GUARD_END
}

int pc_kernel_scalar_mul(const pc_tensor* x, float scalar, const pc_tensor* out, pc_kernel** kernel) {
    PC_GUARD_BEGIN
    return wrap(std::make_unique<UnaryKernel>(launch::Unary::kScalarMul, tensor_arg(x, "x"), tensor_arg(out, "out"),
                                              scalar),
                kernel);
    PC_GUARD_END
}

int pc_kernel_attention_mask_build(const pc_tensor* mask, int32_t sliding_window, pc_kernel** kernel) {
    PC_GUARD_BEGIN
    return wrap(std::make_unique<AttentionMaskBuildKernel>(tensor_arg(mask, "mask"), sliding_window), kernel);
    PC_GUARD_END
}

int pc_kernel_mul(const pc_tensor* a, const pc_tensor* b, const pc_tensor* out, pc_kernel** kernel) {
    PC_GUARD_BEGIN
    return wrap(std::make_unique<BinaryKernel>(launch::Binary::kMul, tensor_arg(a, "a"), tensor_arg(b, "b"),
                                               tensor_arg(out, "out")),
                kernel);
    PC_GUARD_END
}

int pc_kernel_add(const pc_tensor* a, const pc_tensor* b, const pc_tensor* out, pc_kernel** kernel) {
    PC_GUARD_BEGIN
    return wrap(std::make_unique<BinaryKernel>(launch::Binary::kAdd, tensor_arg(a, "a"), tensor_arg(b, "b"),
                                               tensor_arg(out, "out")),
                kernel);
    PC_GUARD_END
}

int pc_kernel_rmsnorm_matmul(const pc_tensor* x, const pc_tensor* norm_weight, float eps, int32_t add_one_to_weight,
                             const pc_tensor* w, const pc_tensor* out, pc_kernel** kernel) {
    PC_GUARD_BEGIN
    Tensor nw;
    if (norm_weight) nw = tensor_arg(norm_weight, "norm_weight");
    return wrap(make_rmsnorm_matmul(tensor_arg(x, "x"), norm_weight ? &nw : nullptr, eps, add_one_to_weight != 0,
                                    tensor_arg(w, "w"), tensor_arg(out, "out")),
                kernel);
    PC_GUARD_END
}

int pc_kernel_gated_mlp(const pc_tensor* x, const pc_tensor* norm_weight, float eps, int32_t add_one_to_weight,
                        const pc_tensor* w_gate, const pc_tensor* w_up, int32_t activation, const pc_tensor* out,
                        pc_kernel** kernel) {
    PC_GUARD_BEGIN
    Tensor nw;
    if (norm_weight) nw = tensor_arg(norm_weight, "norm_weight");
    return wrap(make_gated_mlp(tensor_arg(x, "x"), norm_weight ? &nw : nullptr, eps, add_one_to_weight != 0,
                               tensor_arg(w_gate, "w_gate"), tensor_arg(w_up, "w_up"), activation,
                               tensor_arg(out, "out")),
                kernel);
    PC_GUARD_END
}

int pc_kernel_matmul_residual(const pc_tensor* a, const pc_tensor* w, const pc_tensor* residual, const pc_tensor* out,
                              pc_kernel** kernel) {
    PC_GUARD_BEGIN
    return wrap(make_matmul_residual(tensor_arg(a, "a"), tensor_arg(w, "w"), tensor_arg(residual, "residual"),
                                     tensor_arg(out, "out")),
                kernel);
    PC_GUARD_END
}

int pc_kernel_qkv_projection(const pc_tensor* x, const pc_tensor* norm_weight, float eps, int32_t add_one_to_weight,
                             const pc_tensor* w_qkv, const pc_tensor* q_out, const pc_tensor* k_cache,
                             const pc_tensor* v_cache, int64_t offset, const pc_tensor* position, pc_kernel** kernel) {
    PC_GUARD_BEGIN
    Tensor nw, pos;
    if (norm_weight) nw = tensor_arg(norm_weight, "norm_weight");
    if (position) pos = tensor_arg(position, "position");
    return wrap(make_qkv(tensor_arg(x, "x"), norm_weight ? &nw : nullptr, eps, add_one_to_weight != 0,
                         tensor_arg(w_qkv, "w_qkv"), tensor_arg(q_out, "q_out"), tensor_arg(k_cache, "k_cache"),
                         tensor_arg(v_cache, "v_cache"), offset, position ? &pos : nullptr),
                kernel);
    PC_GUARD_END
}

int pc_kernel_argmax(const pc_tensor* x, const pc_tensor* indices, int32_t axis, pc_kernel** kernel) {
    PC_GUARD_BEGIN
    return wrap(std::make_unique<ArgmaxKernel>(tensor_arg(x, "x"), tensor_arg(indices, "indices"), axis), kernel);
    PC_GUARD_END
}

int pc_kernel_qkv_scatter(const pc_tensor* qkv, const pc_tensor* q_out, const pc_tensor* k_cache,
                          const pc_tensor* v_cache, int64_t offset, const pc_tensor* position, pc_kernel** kernel) {
    PC_GUARD_BEGIN
    Tensor pos;
    if (position) pos = tensor_arg(position, "position");
    return wrap(std::make_unique<QKVScatterKernel>(tensor_arg(qkv, "qkv"), tensor_arg(q_out, "q_out"),
                                                   tensor_arg(k_cache, "k_cache"), tensor_arg(v_cache, "v_cache"),
                                                   offset, position ? &pos : nullptr),
                kernel);
    PC_GUARD_END
}

int pc_kernel_gated_activation(const pc_tensor* gate_up, int32_t activation, const pc_tensor* out,
                               pc_kernel** kernel) {
    PC_GUARD_BEGIN
    return wrap(std::make_unique<GatedActivationKernel>(tensor_arg(gate_up, "gate_up"), activation,
                                                        tensor_arg(out, "out")),
                kernel);
    PC_GUARD_END
}

int pc_kernel_matmul_affine_quantized(const pc_tensor* a, const pc_tensor* packed, const pc_tensor* scales,
                                      const pc_tensor* biases, int64_t out_features, int64_t in_features,
                                      int32_t bits, int32_t group_size, const pc_tensor* c, pc_kernel** kernel) {
    PC_GUARD_BEGIN
    Tensor b;
    if (biases) b = tensor_arg(biases, "biases");
    return wrap(std::make_unique<AqMatmulKernel>(tensor_arg(a, "a"), tensor_arg(packed, "packed"),
                                                 tensor_arg(scales, "scales"), biases ? &b : nullptr, out_features,
                                                 in_features, bits, group_size, tensor_arg(c, "c")),
                kernel);
    PC_GUARD_END
}

int pc_kernel_aq_rmsnorm_matmul(const pc_tensor* x, const pc_tensor* norm_weight, float eps,
                                int32_t add_one_to_weight, const pc_affine_quantized* w, const pc_tensor* out,
                                pc_kernel** kernel) {
    PC_GUARD_BEGIN
    Tensor nw;
    if (norm_weight) nw = tensor_arg(norm_weight, "norm_weight");
    return wrap(std::make_unique<AqFusedKernel>(AqFusedKernel::kNormMatmul, tensor_arg(x, "x"), norm_weight ? &nw : nullptr,
                                                eps, add_one_to_weight != 0, aq_weight_arg(w, "w"),
                                                tensor_arg(out, "out"), nullptr, 0, nullptr, nullptr, 0, nullptr),
                kernel);
    PC_GUARD_END
}

int pc_kernel_aq_matmul_residual(const pc_tensor* x, const pc_affine_quantized* w, const pc_tensor* residual,
                                 const pc_tensor* out, pc_kernel** kernel) {
    PC_GUARD_BEGIN
    Tensor r = tensor_arg(residual, "residual");
    return wrap(std::make_unique<AqFusedKernel>(AqFusedKernel::kResidual, tensor_arg(x, "x"), nullptr, 0.f, false,
                                                aq_weight_arg(w, "w"), tensor_arg(out, "out"), &r, 0, nullptr,
                                                nullptr, 0, nullptr),
                kernel);
    PC_GUARD_END
}

int pc_kernel_aq_gated_mlp(const pc_tensor* x, const pc_tensor* norm_weight, float eps, int32_t add_one_to_weight,
                           const pc_affine_quantized* w_gate_up, int32_t activation, const pc_tensor* out,
                           pc_kernel** kernel) {
    PC_GUARD_BEGIN
    Tensor nw;
    if (norm_weight) nw = tensor_arg(norm_weight, "norm_weight");
    return wrap(std::make_unique<AqFusedKernel>(AqFusedKernel::kGated, tensor_arg(x, "x"), norm_weight ? &nw : nullptr,
                                                eps, add_one_to_weight != 0, aq_weight_arg(w_gate_up, "w_gate_up"),
                                                tensor_arg(out, "out"), nullptr, activation, nullptr, nullptr, 0,
                                                nullptr),
                kernel);
    PC_GUARD_END
}

int pc_kernel_aq_qkv_projection(const pc_tensor* x, const pc_tensor* norm_weight, float eps,
                                int32_t add_one_to_weight, const pc_affine_quantized* w_qkv, const pc_tensor* q_out,
                                const pc_tensor* k_cache, const pc_tensor* v_cache, int64_t offset,
                                const pc_tensor* position, pc_kernel** kernel) {
    PC_GUARD_BEGIN
    Tensor nw, pos;
    if (norm_weight) nw = tensor_arg(norm_weight, "norm_weight");
    if (position) pos = tensor_arg(position, "position");
    Tensor kc = tensor_arg(k_cache, "k_cache"), vc = tensor_arg(v_cache, "v_cache");
    return wrap(std::make_unique<AqFusedKernel>(AqFusedKernel::kQKV, tensor_arg(x, "x"), norm_weight ? &nw : nullptr,
                                                eps, add_one_to_weight != 0, aq_weight_arg(w_qkv, "w_qkv"),
                                                tensor_arg(q_out, "q_out"), nullptr, 0, &kc, &vc, offset,
                                                position ? &pos : nullptr),
                kernel);
    PC_GUARD_END
}

int pc_kernel_embedding_gather(const pc_tensor* ids, const pc_tensor* table, const pc_tensor* out,
                               pc_kernel** kernel) {
    PC_GUARD_BEGIN
    return wrap(std::make_unique<EmbeddingGatherKernel>(tensor_arg(ids, "ids"), tensor_arg(table, "table"),
                                                        tensor_arg(out, "out")),
                kernel);
    PC_GUARD_END
}

int pc_kernel_embedding_gather_affine_quantized(const pc_tensor* ids, const pc_tensor* packed,
                                                const pc_tensor* scales, const pc_tensor* biases, int64_t vocab,
                                                int64_t hidden, int32_t bits, int32_t group_size,
                                                const pc_tensor* out, pc_kernel** kernel) {
    PC_GUARD_BEGIN
    Tensor b;
    if (biases) b = tensor_arg(biases, "biases");
    return wrap(std::make_unique<EmbeddingGatherKernel>(tensor_arg(ids, "ids"), tensor_arg(packed, "packed"),
                                                        tensor_arg(scales, "scales"), biases ? &b : nullptr, vocab,
                                                        hidden, bits, group_size, tensor_arg(out, "out")),
                kernel);
    PC_GUARD_END
}

int pc_kernel_rope_build_cos_sin(const pc_tensor* positions, const pc_tensor* inv_freq, const pc_tensor* cos_out,
                                 const pc_tensor* sin_out, float attention_scaling, pc_kernel** kernel) {
    PC_GUARD_BEGIN
    return wrap(std::make_unique<RopeBuildCosSinKernel>(tensor_arg(positions, "positions"),
                                                        tensor_arg(inv_freq, "inv_freq"), tensor_arg(cos_out, "cos_out"),
                                                        tensor_arg(sin_out, "sin_out"), attention_scaling),
                kernel);
    PC_GUARD_END
}

int pc_kernel_rope_apply(const pc_tensor* x, const pc_tensor* cos_t, const pc_tensor* sin_t, const pc_tensor* out,
                         pc_kernel** kernel) {
    PC_GUARD_BEGIN
    return wrap(std::make_unique<RopeApplyKernel>(tensor_arg(x, "x"), tensor_arg(cos_t, "cos"),
                                                  tensor_arg(sin_t, "sin"), tensor_arg(out, "out")),
                kernel);
    PC_GUARD_END
}

int pc_kernel_qk_norm_rope(const pc_tensor* q, const pc_tensor* k_cache, const pc_tensor* v_cache,
                           const pc_tensor* q_norm, const pc_tensor* k_norm, const pc_tensor* cos_t,
                           const pc_tensor* sin_t, float eps, int32_t add_one_to_weight, int32_t norm_v,
                           int64_t offset, const pc_tensor* position, pc_kernel** kernel) {
    PC_GUARD_BEGIN
    Tensor pos;
    if (position) pos = tensor_arg(position, "position");
    return wrap(std::make_unique<QKNormRopeKernel>(tensor_arg(q, "q"), tensor_arg(k_cache, "k_cache"),
                                                   tensor_arg(v_cache, "v_cache"), tensor_arg(q_norm, "q_norm"),
                                                   tensor_arg(k_norm, "k_norm"), tensor_arg(cos_t, "cos"),
                                                   tensor_arg(sin_t, "sin"), eps, add_one_to_weight != 0, norm_v != 0,
                                                   offset, position ? &pos : nullptr),
                kernel);
    PC_GUARD_END
}

int pc_kernel_add_rmsnorm(const pc_tensor* a, const pc_tensor* b, const pc_tensor* norm_weight, float eps,
                          int32_t add_one_to_weight, const pc_tensor* sum_out, const pc_tensor* norm_out,
                          pc_kernel** kernel) {
    PC_GUARD_BEGIN
    Tensor nw;
    if (norm_weight) nw = tensor_arg(norm_weight, "norm_weight");
    return wrap(std::make_unique<AddRMSNormKernel>(tensor_arg(a, "a"), tensor_arg(b, "b"),
                                                   norm_weight ? &nw : nullptr, eps, add_one_to_weight != 0,
                                                   tensor_arg(sum_out, "sum_out"), tensor_arg(norm_out, "norm_out")),
                kernel);
    PC_GUARD_END
}

int pc_kernel_allreduce_add_rmsnorm(const pc_peer_group* group, int32_t buffer, const pc_tensor* residual,
                                    const pc_tensor* norm_weight, float eps, int32_t add_one_to_weight,
                                    const pc_tensor* sum_out, const pc_tensor* norm_out, pc_kernel** kernel) {
    PC_GUARD_BEGIN
    Tensor nw;
    if (norm_weight) nw = tensor_arg(norm_weight, "norm_weight");
    return wrap(std::make_unique<PeerAllReduceKernel>(group, buffer, tensor_arg(residual, "residual"),
                                                      norm_weight ? &nw : nullptr, eps, add_one_to_weight != 0,
                                                      tensor_arg(sum_out, "sum_out"), tensor_arg(norm_out, "norm_out")),
                kernel);
    PC_GUARD_END
}

int pc_kernel_matmul_allreduce_add_rmsnorm(const pc_tensor* a, const pc_tensor* w, const pc_peer_group* group,
                                           int32_t buffer, const pc_tensor* residual, const pc_tensor* norm_weight,
                                           float eps, int32_t add_one_to_weight, const pc_tensor* sum_out,
                                           const pc_tensor* norm_out, pc_kernel** kernel) {
    PC_GUARD_BEGIN
    Tensor nw;
    if (norm_weight) nw = tensor_arg(norm_weight, "norm_weight");
    return wrap(std::make_unique<MatmulAllReduceKernel>(tensor_arg(a, "a"), tensor_arg(w, "w"), group, buffer,
                                                        tensor_arg(residual, "residual"), norm_weight ? &nw : nullptr,
                                                        eps, add_one_to_weight != 0, tensor_arg(sum_out, "sum_out"),
                                                        tensor_arg(norm_out, "norm_out")),
                kernel);
    PC_GUARD_END
}

int pc_decode_stack_workspace_bytes(const pc_decode_stack_desc* desc, uint64_t* bytes) {
    try {
        launch::DecodeStep p = make_step(desc);
        *bytes = launch::decode_step_workspace_bytes(p);
    } catch (const PopcornError& e) {
        set_last_error(e.message);
        return e.code;
    }
    return PC_OK;
}

int pc_kernel_decode_stack(const pc_decode_stack_desc* desc, pc_kernel** kernel) {
    PC_GUARD_BEGIN
    return wrap(std::make_unique<DecodeStackKernel>(desc), kernel);
    PC_GUARD_END
}

}  // extern "C"
