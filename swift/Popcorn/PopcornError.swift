// PopcornError over the C ABI (reference: Sources/Popcorn/PopcornError.swift:23-58).
// The numeric codes are the ABI's pc_status values, which are the reference's
// PopcornError.Code raw values; the message is the ABI's thread-local
// pc_last_error_message().
import PopcornCUDA

public struct PopcornError: Error, CustomStringConvertible {
    public enum Code: Int32 {
        case constantAllocationFailed = -1001
        case tensorAllocationFailed = -1003
        case kernelFunctionNotFound = -1006
        case tensorShapeMismatch = -1007
        case tensorInvalidRank = -1008
        case tensorInvalidAxis = -1009
        case unsupportedDataTypeCombination = -1010
        case workspaceExhausted = -1012
        case gpuOutOfMemory = -1013
        case gpuTimeout = -1014
        case gpuPageFault = -1015
        case gpuInvalidResource = -1016
        case gpuDeviceRemoved = -1017
        case gpuAccessRevoked = -1018
        case gpuInternal = -1019
    }

    public let code: Code
    public let message: String

    public var description: String { "PopcornError(\(code.rawValue)): \(message)" }
}

/// Turns an ABI status into a thrown PopcornError (0 returns normally).
@inline(__always)
func check(_ status: Int32) throws {
    guard status != 0 else { return }
    let message = String(cString: pc_last_error_message())
    throw PopcornError(code: PopcornError.Code(rawValue: status) ?? .gpuInternal, message: message)
}
