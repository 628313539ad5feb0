// Scratch protocol (reference: Sources/Popcorn/KernelResources.swift:5-36).
// Composite kernels (split-KV decode attention, Argmax over long rows, the
// split-K GEMM) borrow temporary device buffers while they are encoded and
// release them when encoding ends; stream order protects later reuse.
public struct KernelTemporaryBuffer {
    public let pointer: UnsafeMutableRawPointer
    public let length: Int
    public let wasReused: Bool

    public init(pointer: UnsafeMutableRawPointer, length: Int, wasReused: Bool = false) {
        self.pointer = pointer
        self.length = length
        self.wasReused = wasReused
    }
}

public protocol KernelScratchAllocator: AnyObject {
    func borrowTemporaryBuffer(length: Int) throws -> KernelTemporaryBuffer
    func releaseTemporaryBuffer(_ temporary: KernelTemporaryBuffer)
}
