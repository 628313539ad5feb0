// KernelLibrary over the C ABI (reference: Sources/Popcorn/KernelLibrary.swift:4-41).
// The ABI's library is thread-safe (the reference guards its pipeline cache
// with a lock); lookups of the same name return the same handle.
import PopcornCUDA

public final class KernelLibrary {
    let handle: OpaquePointer
    public let device: Int32

    public init(device: Int32 = 0) throws {
        var h: OpaquePointer?
        try check(pc_library_create(device, &h))
        handle = h!
        self.device = device
    }

    deinit { pc_library_destroy(handle) }

    /// The launchable function registered under `name` (the reference's
    /// pipelineState(for:)); unknown names throw .kernelFunctionNotFound.
    public func pipelineState(for name: String) throws -> UnsafeRawPointer {
        var p: UnsafeRawPointer?
        try check(pc_library_lookup(handle, name, &p))
        return p!
    }

    public var functionNames: [String] {
        (0..<Int(pc_library_function_count(handle))).map {
            String(cString: pc_library_function_name(handle, Int32($0)))
        }
    }
}
