// Tensor over a caller-owned device pointer (reference: Sources/Popcorn/Tensor.swift:5-218).
// The reference wraps an MTLBuffer; here the buffer is a CUDA device pointer
// (from pc_buffer_alloc or any other allocator). The library never frees it.
import PopcornCUDA

public struct Tensor {
    public let pointer: UnsafeMutableRawPointer
    public let shape: Shape
    public let dataType: DataType

    public init(pointer: UnsafeMutableRawPointer, shape: Shape, dataType: DataType = .f32) {
        self.pointer = pointer
        self.shape = shape
        self.dataType = dataType
    }

    public init(pointer: UnsafeMutableRawPointer, shape: [Int], dataType: DataType = .f32) {
        self.init(pointer: pointer, shape: Shape(shape), dataType: dataType)
    }

    /// The ABI descriptor (pc_tensor) of this tensor.
    var descriptor: pc_tensor {
        var t = pc_tensor()
        t.data = pointer
        t.dtype = Int32(dataType.rawValue)
        t.rank = Int32(shape.rank)
        withUnsafeMutableBytes(of: &t.shape) { raw in
            let dims = raw.bindMemory(to: Int64.self)
            for (i, d) in shape.dimensions.enumerated() { dims[i] = Int64(d) }
        }
        return t
    }
}

public extension Tensor {
    struct Shape: ExpressibleByArrayLiteral, Equatable {
        public var dimensions: [Int]
        public init(_ dimensions: [Int]) { self.dimensions = dimensions }
        public init(arrayLiteral elements: Int...) { dimensions = elements }
        public var rank: Int { dimensions.count }
        public var elementCount: Int { dimensions.reduce(1, *) }
        public subscript(index: Int) -> Int { dimensions[index] }
    }

    /// Same order as the reference (and as pc_dtype).
    enum DataType: UInt8 {
        case u8, u16, u32, u64, i8, i16, i32, i64, f32, f16, bf16

        public var stride: Int { Int(pc_dtype_stride(Int32(rawValue))) }
    }

    struct Access: OptionSet {
        public let rawValue: UInt8
        public init(rawValue: UInt8) { self.rawValue = rawValue }
        public static let read = Access(rawValue: 1 << 0)
        public static let write = Access(rawValue: 1 << 1)
        public static let readWrite: Access = [.read, .write]
    }

    struct Binding {
        public let tensor: Tensor
        public let access: Access
        public init(tensor: Tensor, access: Access) {
            self.tensor = tensor
            self.access = access
        }
    }
}
