// Backend selection: CUDA in the plugin slot MetalBackend occupies
// (TinyBrainBackend.metalBackend, Sources/TinyBrainRuntime/Backend.swift:29),
// registered the way Sources/TinyBrain/TinyBrain.swift:35-100 registers Metal.
// Every QuantizedMatMulBackend / AttentionBackend dispatch of the runtime then
// reaches CUDABackend; CUDAModelRunner takes whole decode steps.
//
// Written against the reference's public API; not built in this repository.
import Foundation
import TinyBrainRuntime

extension TinyBrainBackend {
    /// The CUDA backend in the slot, if enableCUDA() installed one.
    public static var cudaBackend: CUDABackend? { metalBackend as? CUDABackend }

    /// Install CUDABackend (device `device`) as the GPU backend.  Returns false
    /// when no CUDA device is visible or the context cannot be created.
    @discardableResult
    public static func enableCUDA(device: Int32 = 0) -> Bool {
        if metalBackend is CUDABackend { return true }
        guard CUDABackend.isAvailable else {
            if debugLogging { print("[TinyBrain] no CUDA device") }
            return false
        }
        do {
            metalBackend = try CUDABackend(device: device)
            if debugLogging { print("[TinyBrain] CUDA (B200) backend enabled") }
            return true
        } catch {
            if debugLogging { print("[TinyBrain] CUDA initialization failed: \(error)") }
            return false
        }
    }

    /// A decode runner on the CUDA backend for `weights` (the whole step on
    /// the device), enabling the backend first if needed.
    public static func makeCUDARunner(weights: ModelWeights) throws -> CUDAModelRunner {
        guard enableCUDA(), let backend = cudaBackend else {
            throw CUDABackendError.unsupported("no CUDA backend")
        }
        return try CUDAModelRunner(weights: weights, backend: backend)
    }
}
