// CUDABackend -- the op-level plugin: libtinybrain_cuda behind TinyBrain's
// backend protocols (Sources/TinyBrainRuntime/Backend.swift:158-228), in the
// slot MetalBackend fills today (TinyBrainBackend.metalBackend, Backend.swift:29).
//
// QuantizedMatMulBackend.matmulQuantized (Backend.swift:173-175; Metal:
// MetalBackend.swift:894-1048) uploads each QuantizedTensor once, keyed by its
// identifier (the role of MetalBackend.cachedQuantizedBuffers), and runs the
// B200 dequantising GEMV (tb_matmul_quantized).  AttentionBackend.attention
// (Backend.swift:205-219) runs single-query decode attention
// (tb_attention_decode); other shapes and masks throw, and the reference's
// dispatch helpers then take their CPU path, as they do for a failing Metal
// call.  Errors carry tb_last_error(); there is no silent fallback inside.
//
// This file is written against the reference's public API; it is not built in
// this repository (no Swift toolchain on Linux CUDA hosts here).
import CTinyBrainCUDA
import Foundation
import TinyBrainRuntime

public enum CUDABackendError: Error, CustomStringConvertible {
    case library(status: Int32, message: String)
    case unsupported(String)

    public var description: String {
        switch self {
        case let .library(status, message):
            let name = String(cString: tb_status_string(tb_status(rawValue: UInt32(status))))
            return "libtinybrain_cuda: \(name): \(message)"
        case let .unsupported(what):
            return "libtinybrain_cuda: unsupported: \(what)"
        }
    }
}

/// Throws on a non-TB_OK status with the calling thread's last error message.
@inline(__always)
func tbCheck(_ status: tb_status) throws {
    guard status == TB_OK else {
        throw CUDABackendError.library(status: Int32(status.rawValue), message: String(cString: tb_last_error()))
    }
}

/// QuantizedTensor (QuantizedTensor.swift:62-165) as the C descriptor; the
/// closure runs while the arrays are pinned.
func withQTensorDesc<R>(_ q: QuantizedTensor, _ body: (UnsafePointer<tb_qtensor_desc>) throws -> R) rethrows -> R {
    let dims = q.shape.dimensions
    return try q.data.withUnsafeBytes { dataBuf in
        try q.scales.withUnsafeBufferPointer { scaleBuf in
            func finish(_ zp: UnsafeBufferPointer<Int8>?) throws -> R {
                var d = tb_qtensor_desc()
                d.precision = q.precision == .int4 ? Int32(TB_PREC_INT4.rawValue) : Int32(TB_PREC_INT8.rawValue)
                d.in_features = Int64(dims[0])
                d.out_features = Int64(dims[1])
                d.group_size = Int64(q.groupSize)
                d.data = dataBuf.baseAddress
                d.data_bytes = Int64(dataBuf.count)
                d.scales = scaleBuf.baseAddress
                d.num_scales = Int64(scaleBuf.count)
                d.zero_points = zp?.baseAddress
                d.num_zero_points = Int64(zp?.count ?? 0)
                return try withUnsafePointer(to: &d) { try body($0) }
            }
            if let zps = q.zeroPoints {
                return try zps.withUnsafeBufferPointer { try finish($0) }
            }
            return try finish(nil)
        }
    }
}

public final class CUDABackend: QuantizedMatMulBackend, AttentionBackend {
    let ctx: OpaquePointer
    private var weights: [UUID: OpaquePointer] = [:]  // QuantizedTensor.identifier -> tb_qweight
    private let lock = NSLock()

    /// One context per GPU (replaces MetalBackend.init, MetalBackend.swift:56-108).
    public init(device: Int32 = 0) throws {
        var c: OpaquePointer?
        try tbCheck(tb_context_create(device, &c))
        guard let c else { throw CUDABackendError.unsupported("no context") }
        ctx = c
    }

    deinit {
        for w in weights.values { tb_qweight_free(w) }
        tb_context_destroy(ctx)
    }

    public static var isAvailable: Bool {
        var n: Int32 = 0
        return tb_device_count(&n) == TB_OK && n > 0
    }

    private func uploaded(_ q: QuantizedTensor) throws -> OpaquePointer {
        lock.lock()
        defer { lock.unlock() }
        if let w = weights[q.identifier] { return w }
        var w: OpaquePointer?
        try withQTensorDesc(q) { try tbCheck(tb_qweight_upload(ctx, $0, &w)) }
        guard let w else { throw CUDABackendError.unsupported("weight upload") }
        weights[q.identifier] = w
        return w
    }

    /// y[M][N] = x[M][K] * dequant(W[K][N]) (QuantizedTensor.swift:627-643).
    public func matmulQuantized(_ input: Tensor<Float>, _ quantized: QuantizedTensor) throws -> Tensor<Float> {
        let dims = input.shape.dimensions
        let K = quantized.shape.dimensions[0], N = quantized.shape.dimensions[1]
        let M = dims.count == 1 ? 1 : dims.dropLast().reduce(1, *)
        guard dims.last == K else { throw CUDABackendError.unsupported("input width \(dims) vs K = \(K)") }
        let w = try uploaded(quantized)
        var out = [Float](repeating: 0, count: M * N)
        try input.scalars.withUnsafeBufferPointer { x in
            try out.withUnsafeMutableBufferPointer { y in
                try tbCheck(tb_matmul_quantized(ctx, x.baseAddress, Int64(M), w, y.baseAddress))
            }
        }
        return Tensor(shape: TensorShape(dims.count == 1 ? [N] : Array(dims.dropLast()) + [N]), data: out)
    }

    /// Decode attention for one query token over a contiguous cache
    /// (ModelRunner.swift:519-579 semantics).
    public func attention(query: Tensor<Float>, keys: Tensor<Float>, values: Tensor<Float>,
                          mask: Tensor<Float>?, headDim: Int, numHeads: Int, numKVHeads: Int) throws -> Tensor<Float> {
        guard mask == nil else { throw CUDABackendError.unsupported("attention mask") }
        guard query.scalars.count == numHeads * headDim else {
            throw CUDABackendError.unsupported("more than one query token")
        }
        let L = keys.scalars.count / (numKVHeads * headDim)
        var out = [Float](repeating: 0, count: numHeads * headDim)
        try query.scalars.withUnsafeBufferPointer { q in
            try keys.scalars.withUnsafeBufferPointer { k in
                try values.scalars.withUnsafeBufferPointer { v in
                    try out.withUnsafeMutableBufferPointer { o in
                        try tbCheck(tb_attention_decode(ctx, q.baseAddress, k.baseAddress, v.baseAddress, Int64(L),
                                                        Int32(numHeads), Int32(numKVHeads), Int32(headDim),
                                                        o.baseAddress))
                    }
                }
            }
        }
        return Tensor(shape: query.shape, data: out)
    }
}
