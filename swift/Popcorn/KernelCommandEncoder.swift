// KernelCommandEncoder over the C ABI (reference:
// Sources/Popcorn/KernelCommandEncoder.swift:8-168). The ABI encoder does the
// reference's bookkeeping (dispatch sequencing, hazard tracking keyed by
// buffer address, scratch borrowing); this class bridges the Swift scratch
// allocator to the ABI's C callbacks. As with the reference, the caller owns
// the stream (the command buffer's role): encode() only enqueues, and the
// caller synchronises.
import PopcornCUDA

/// Holds the Swift allocator and the buffers it has lent to the ABI, so the
/// C release callback (which only sees a device pointer) can hand back the
/// exact KernelTemporaryBuffer that was borrowed.
final class ScratchBridge {
    let allocator: any KernelScratchAllocator
    var live: [UnsafeMutableRawPointer: [KernelTemporaryBuffer]] = [:]

    init(_ allocator: any KernelScratchAllocator) { self.allocator = allocator }

    func borrow(_ length: Int) -> KernelTemporaryBuffer? {
        guard let t = try? allocator.borrowTemporaryBuffer(length: length) else { return nil }
        live[t.pointer, default: []].append(t)
        return t
    }

    func release(_ pointer: UnsafeMutableRawPointer) {
        guard var lent = live[pointer], let t = lent.popLast() else { return }
        live[pointer] = lent.isEmpty ? nil : lent
        allocator.releaseTemporaryBuffer(t)
    }
}

private func bridge(_ ctx: UnsafeMutableRawPointer?) -> ScratchBridge {
    Unmanaged<ScratchBridge>.fromOpaque(ctx!).takeUnretainedValue()
}

public final class KernelCommandEncoder {
    let handle: OpaquePointer
    public let library: KernelLibrary
    private let scratch: Unmanaged<ScratchBridge>?

    /// `stream` is a cudaStream_t (nil: the legacy default stream).
    public init(stream: UnsafeMutableRawPointer?, library: KernelLibrary,
                scratch: (any KernelScratchAllocator)? = nil) throws {
        self.library = library
        var h: OpaquePointer?
        if let scratch {
            let box = Unmanaged.passRetained(ScratchBridge(scratch))
            var alloc = pc_scratch_allocator(
                ctx: box.toOpaque(),
                borrow: { ctx, length, out, reused in
                    guard let t = bridge(ctx).borrow(Int(length)) else {
                        return PopcornError.Code.tensorAllocationFailed.rawValue
                    }
                    out!.pointee = t.pointer
                    reused!.pointee = t.wasReused ? 1 : 0
                    return 0
                },
                release: { ctx, pointer in
                    if let pointer { bridge(ctx).release(pointer) }
                })
            let status = pc_encoder_create(library.handle, stream, &alloc, &h)
            if status != 0 { box.release() }
            try check(status)
            self.scratch = box
        } else {
            try check(pc_encoder_create(library.handle, stream, nil, &h))
            self.scratch = nil
        }
        handle = h!
    }

    deinit {
        pc_encoder_destroy(handle)
        scratch?.release()
    }

    /// encode(_:), KernelCommandEncoder.swift:39-47.
    public func encode(_ kernels: any Kernel...) throws {
        for k in kernels { try check(pc_encoder_encode(handle, k.handle)) }
    }

    /// barrier(), KernelCommandEncoder.swift:71-85 (a bookkeeping reset on
    /// one CUDA stream, where launches are already ordered).
    public func barrier() { _ = pc_encoder_barrier(handle) }

    public var barrierCount: Int64 { pc_encoder_barrier_count(handle) }
    public var dispatchCount: Int64 { pc_encoder_dispatch_count(handle) }
}
