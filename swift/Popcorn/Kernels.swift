// The reference's kernel value types over the C ABI (reference:
// Sources/Popcorn/Kernel.swift:15-19 and Sources/Popcorn/Kernels/*.swift).
// Each initialiser validates through the ABI (which throws the reference's
// error codes before anything launches) and keeps the kernel handle;
// routing stays hidden behind one semantic type, as in the reference.
import PopcornCUDA

public enum Kernels {}

public protocol Kernel {
    var handle: OpaquePointer { get }
}

/// Owns one pc_kernel handle.
public final class KernelHandle {
    let raw: OpaquePointer
    init(_ raw: OpaquePointer) { self.raw = raw }
    deinit { pc_kernel_destroy(raw) }
}

public extension Kernel {
    /// The functions this kernel launches (its route made visible).
    var functionNames: [String] {
        String(cString: pc_kernel_function_names(handle)).split(separator: ";").map(String.init)
    }
}

/// AttentionMask, Sources/Popcorn/Kernels/AttentionMask.swift:17-41.
public enum AttentionMask {
    case causal
    case causalSlidingWindow(Int)
    case bidirectional

    var descriptor: pc_attention_mask {
        switch self {
        case .causal: return pc_attention_mask(kind: 0, window: -1)
        case let .causalSlidingWindow(w): return pc_attention_mask(kind: 1, window: Int32(w))
        case .bidirectional: return pc_attention_mask(kind: 2, window: -1)
        }
    }
}

/// Runs an ABI constructor and wraps the handle it returns.
private func make(_ body: (UnsafeMutablePointer<OpaquePointer?>) -> Int32) throws -> KernelHandle {
    var h: OpaquePointer?
    try check(body(&h))
    return KernelHandle(h!)
}

public extension Kernels {
    /// FlashAttention.swift:51-90; Sq == 1 routes to split-KV decoding.
    struct FlashAttention: Kernel {
        let owner: KernelHandle
        public var handle: OpaquePointer { owner.raw }
        public init(q: Tensor, k: Tensor, v: Tensor, into out: Tensor, scale: Float,
                    mask: AttentionMask = .causal) throws {
            var (cq, ck, cv, co) = (q.descriptor, k.descriptor, v.descriptor, out.descriptor)
            owner = try make { pc_kernel_flash_attention(&cq, &ck, &cv, &co, scale, mask.descriptor, $0) }
        }
    }

    /// KVCacheWrite.swift:38-49.
    struct KVCacheWrite: Kernel {
        let owner: KernelHandle
        public var handle: OpaquePointer { owner.raw }
        public init(source: Tensor, cache: Tensor, offset: Int) throws {
            var (cs, cc) = (source.descriptor, cache.descriptor)
            owner = try make { pc_kernel_kv_cache_write(&cs, &cc, Int64(offset), $0) }
        }
    }

    /// RMSNorm.swift:39-70 (weight is f32 [H], or nil).
    struct RMSNorm: Kernel {
        let owner: KernelHandle
        public var handle: OpaquePointer { owner.raw }
        public init(_ x: Tensor, weight: Tensor?, into out: Tensor, axis: Int = -1, eps: Float = 1e-6,
                    addOneToWeight: Bool = false) throws {
            var (cx, co) = (x.descriptor, out.descriptor)
            if var cw = weight?.descriptor {
                owner = try make { pc_kernel_rmsnorm(&cx, &cw, &co, Int32(axis), eps, addOneToWeight ? 1 : 0, $0) }
            } else {
                owner = try make { pc_kernel_rmsnorm(&cx, nil, &co, Int32(axis), eps, addOneToWeight ? 1 : 0, $0) }
            }
        }
    }

    /// Matmul.swift:68-93; M == 1 with transposeB routes to the matvec.
    struct Matmul: Kernel {
        let owner: KernelHandle
        public var handle: OpaquePointer { owner.raw }
        public init(_ a: Tensor, _ b: Tensor, into c: Tensor, transposeB: Bool = false) throws {
            var (ca, cb, cc) = (a.descriptor, b.descriptor, c.descriptor)
            owner = try make { pc_kernel_matmul(&ca, &cb, &cc, transposeB ? 1 : 0, $0) }
        }
    }

    /// GeluTanh.swift:8-26.
    struct GeluTanh: Kernel {
        let owner: KernelHandle
        public var handle: OpaquePointer { owner.raw }
        public init(_ x: Tensor, into out: Tensor) throws {
            var (cx, co) = (x.descriptor, out.descriptor)
            owner = try make { pc_kernel_gelu_tanh(&cx, &co, $0) }
        }
    }

    /// Mul.swift.
    struct Mul: Kernel {
        let owner: KernelHandle
        public var handle: OpaquePointer { owner.raw }
        public init(_ a: Tensor, _ b: Tensor, into out: Tensor) throws {
            var (ca, cb, co) = (a.descriptor, b.descriptor, out.descriptor)
            owner = try make { pc_kernel_mul(&ca, &cb, &co, $0) }
        }
    }

    /// Add.swift.
    struct Add: Kernel {
        let owner: KernelHandle
        public var handle: OpaquePointer { owner.raw }
        public init(_ a: Tensor, _ b: Tensor, into out: Tensor) throws {
            var (ca, cb, co) = (a.descriptor, b.descriptor, out.descriptor)
            owner = try make { pc_kernel_add(&ca, &cb, &co, $0) }
        }
    }

    /// Extension: decode attention over a [B,Nkv,Smax,Hd] cache with
    /// per-sequence lengths (pc_kernel_flash_decoding_ragged).
    struct FlashDecodingRagged: Kernel {
        let owner: KernelHandle
        public var handle: OpaquePointer { owner.raw }
        public init(q: Tensor, kCache: Tensor, vCache: Tensor, seqLens: Tensor, into out: Tensor, scale: Float,
                    mask: AttentionMask = .causal) throws {
            var (cq, ck, cv, cl, co) = (q.descriptor, kCache.descriptor, vCache.descriptor, seqLens.descriptor,
                                        out.descriptor)
            owner = try make { pc_kernel_flash_decoding_ragged(&cq, &ck, &cv, &cl, &co, scale, mask.descriptor, $0) }
        }
    }
}
