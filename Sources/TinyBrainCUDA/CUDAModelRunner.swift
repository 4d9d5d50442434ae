// CUDAModelRunner -- the runner-level binding: ModelRunner's public surface
// (Sources/TinyBrainRuntime/ModelRunner.swift:127-298) over tb_runner, so that
// a whole decode step (every layer, attention over the HBM page cache, the LM
// head and the greedy / sampled draw) is one CUDA graph on the device instead
// of one plugin round trip per projection.
//
//   init(weights:)            ModelWeights (ModelWeights.swift:137-168) ->
//                             tb_model_create / tb_model_set_* / tb_model_finalize,
//                             tb_runner_create
//   step(tokenId:)            tb_runner_step (or tb_runner_step_observed while an
//                             InferenceObserver is attached: InferenceObserver.swift:40-84)
//   reset()                   tb_runner_reset
//   generateStream(prompt:config:)
//                             tb_runner_generate with a per-token callback;
//                             SamplerConfig -> tb_sampler_config (tb_runner_set_sampler)
//                             unless it is greedy (topK 1, no penalty), which
//                             stays the LM-head argmax; TokenOutput.probability /
//                             .entropy from tb_runner_token_stats
//   kvCacheLength, pageAllocationStatus()
//                             tb_runner_kv_length, tb_runner_page_status
//
// Written against the reference's public API; not built in this repository.
import CTinyBrainCUDA
import Foundation
import TinyBrainRuntime

public final class CUDAModelRunner {
    public let config: ModelConfig
    public private(set) var currentPosition: Int = 0
    public weak var observer: InferenceObserver?
    private let backend: CUDABackend
    private let model: OpaquePointer
    private let runner: OpaquePointer

    public init(weights: ModelWeights, backend: CUDABackend) throws {
        self.backend = backend
        config = weights.config
        guard !config.isPhiStyle, !config.isGemmaStyle else {
            throw CUDABackendError.unsupported("architecture \(config.architecture)")
        }
        let toy = weights.layers.first?.inputNormWeights == nil
        var c = tb_model_config(num_layers: Int32(config.numLayers), hidden_dim: Int32(config.hiddenDim),
                                num_heads: Int32(config.numHeads), num_kv_heads: Int32(config.numKVHeads),
                                vocab_size: Int32(config.vocabSize), max_seq_len: Int32(config.maxSeqLen),
                                intermediate_dim: Int32(config.intermediateDim),
                                architecture: Int32(toy ? TB_ARCH_TOY.rawValue : TB_ARCH_LLAMA.rawValue),
                                rms_eps: 1e-5)
        var m: OpaquePointer?
        try tbCheck(tb_model_create(backend.ctx, &c, &m))
        guard let m else { throw CUDABackendError.unsupported("model") }
        model = m
        try weights.tokenEmbeddings.scalars.withUnsafeBufferPointer { try tbCheck(tb_model_set_embedding(m, $0.baseAddress)) }
        if let fn = weights.finalNormWeights {
            try fn.scalars.withUnsafeBufferPointer { try tbCheck(tb_model_set_final_norm(m, $0.baseAddress)) }
        }
        func setProjection(_ layer: Int, _ which: tb_projection, _ lw: LinearLayerWeights) throws {
            try withQTensorDesc(lw.weights) { desc in
                if let b = lw.bias {
                    try b.scalars.withUnsafeBufferPointer {
                        try tbCheck(tb_model_set_projection(m, Int32(layer), Int32(which.rawValue), desc, $0.baseAddress))
                    }
                } else {
                    try tbCheck(tb_model_set_projection(m, Int32(layer), Int32(which.rawValue), desc, nil))
                }
            }
        }
        for (i, layer) in weights.layers.enumerated() {
            if let a = layer.inputNormWeights, let b = layer.postAttentionNormWeights {
                try a.scalars.withUnsafeBufferPointer { an in
                    try b.scalars.withUnsafeBufferPointer { bn in
                        try tbCheck(tb_model_set_layer_norms(m, Int32(i), an.baseAddress, bn.baseAddress))
                    }
                }
            }
            try setProjection(i, TB_PROJ_Q, layer.attention.query)
            try setProjection(i, TB_PROJ_K, layer.attention.key)
            try setProjection(i, TB_PROJ_V, layer.attention.value)
            try setProjection(i, TB_PROJ_O, layer.attention.output)
            if let g = layer.feedForward.gate { try setProjection(i, TB_PROJ_GATE, g) }
            try setProjection(i, TB_PROJ_UP, layer.feedForward.up)
            try setProjection(i, TB_PROJ_DOWN, layer.feedForward.down)
        }
        try withQTensorDesc(weights.output.weights) { desc in
            if let b = weights.output.bias {
                try b.scalars.withUnsafeBufferPointer { try tbCheck(tb_model_set_output(m, desc, $0.baseAddress)) }
            } else {
                try tbCheck(tb_model_set_output(m, desc, nil))
            }
        }
        try tbCheck(tb_model_finalize(m))
        var r: OpaquePointer?
        try tbCheck(tb_runner_create(m, 1, Int32(config.maxSeqLen + 64), &r))
        guard let r else { throw CUDABackendError.unsupported("runner") }
        runner = r
    }

    deinit {
        tb_runner_free(runner)
        tb_model_free(model)
    }

    /// ModelRunner.step(tokenId:) (ModelRunner.swift:168-208): logits [vocabSize].
    public func step(tokenId: Int) throws -> Tensor<Float> {
        let V = config.vocabSize
        var logits = [Float](repeating: 0, count: V)
        var argmax: Int32 = 0
        let pos = currentPosition
        if let obs = observer {
            let L = pos + 1, H = config.numHeads
            var norms = [Float](repeating: 0, count: config.numLayers)
            var attn = [Float](repeating: 0, count: config.numLayers * H * L)
            var fin = [Float](repeating: 0, count: config.hiddenDim)
            try tbCheck(tb_runner_step_observed(runner, Int32(tokenId), &logits, &argmax, &norms, &attn,
                                                Int64(H * L), &fin))
            for layer in 0..<config.numLayers {
                obs.didEnterLayer(layerIndex: layer, hiddenStateNorm: norms[layer], position: pos)
                obs.didComputeAttention(layerIndex: layer,
                                        weights: Array(attn[(layer * H * L)..<((layer + 1) * H * L)]), position: pos)
            }
            obs.didComputeFinalHiddenState(fin, position: pos)
            obs.didComputeLogits(logits: logits, position: pos)
        } else {
            try tbCheck(tb_runner_step(runner, Int32(tokenId), &logits, &argmax))
        }
        currentPosition += 1
        return Tensor(shape: TensorShape([V]), data: logits)
    }

    /// ModelRunner.reset() (ModelRunner.swift:213-217).
    public func reset() throws {
        try tbCheck(tb_runner_reset(runner))
        currentPosition = 0
    }

    public var kvCacheLength: Int {
        var n: Int64 = 0
        _ = tb_runner_kv_length(runner, 0, &n)
        return Int(n)
    }

    /// KVCache.pageAllocationStatus() (KVCache.swift:352-356).
    public func pageAllocationStatus() -> [Bool] {
        var n: Int64 = 0
        _ = tb_runner_max_pages(runner, &n)
        var st = [UInt8](repeating: 0, count: Int(n))
        _ = tb_runner_page_status(runner, 0, &st, n)
        return st.map { $0 != 0 }
    }

    private final class TokenSink {
        var tokens: [Int] = []
        let onToken: (Int) -> Void
        init(_ onToken: @escaping (Int) -> Void) { self.onToken = onToken }
    }

    /// ModelRunner.generateStream(prompt:config:) (ModelRunner.swift:227-298):
    /// the prompt is clamped and prefilled and every token drawn on the device.
    public func generateStream(prompt: [Int], config gen: GenerationConfig = GenerationConfig())
        -> AsyncThrowingStream<TokenOutput, Error>
    {
        AsyncThrowingStream { continuation in
            Task {
                do {
                    let sc = gen.sampler
                    let greedy = sc.topK == 1 && sc.repetitionPenalty == 1.0
                    if greedy {
                        try tbCheck(tb_runner_set_sampler(self.runner, nil))
                    } else {
                        var c = tb_sampler_config(temperature: sc.temperature, top_k: Int32(sc.topK ?? 0),
                                                  has_top_p: sc.topP == nil ? 0 : 1, top_p: sc.topP ?? 0,
                                                  repetition_penalty: sc.repetitionPenalty,
                                                  has_seed: sc.seed == nil ? 0 : 1, seed: sc.seed ?? 0)
                        try tbCheck(tb_runner_set_sampler(self.runner, &c))
                    }
                    let ids = prompt.map { Int32(max(0, min($0, self.config.vocabSize - 1))) }
                    var offsets: [Int64] = [0, Int64(ids.count)]
                    let stops = gen.stopTokens.map { Int32($0) }
                    var out = [Int32](repeating: 0, count: max(1, gen.maxTokens))
                    var count: Int32 = 0
                    let sink = TokenSink { _ in }
                    let user = Unmanaged.passUnretained(sink).toOpaque()
                    let cb: tb_token_callback = { user, _, _, token in
                        Unmanaged<TokenSink>.fromOpaque(user!).takeUnretainedValue().tokens.append(Int(token))
                        return 0
                    }
                    try tbCheck(tb_runner_generate(self.runner, ids, &offsets, 1, Int32(gen.maxTokens), stops,
                                                   Int32(stops.count), &out, &count, cb, user))
                    var prob = [Float](repeating: 1.0 / (1.0 + 1e-7), count: max(1, gen.maxTokens))
                    var ent = prob.map { -$0 * log($0) }
                    if !greedy {
                        try tbCheck(tb_runner_token_stats(self.runner, 1, Int32(gen.maxTokens), &prob, &ent))
                        try tbCheck(tb_runner_set_sampler(self.runner, nil))
                    }
                    for (i, t) in sink.tokens.enumerated() {
                        continuation.yield(TokenOutput(tokenId: t, probability: prob[i], entropy: ent[i],
                                                       timestamp: Date(), strategy: nil, energyJoules: nil))
                    }
                    continuation.finish()
                } catch {
                    continuation.finish(throwing: error)
                }
            }
        }
    }
}
