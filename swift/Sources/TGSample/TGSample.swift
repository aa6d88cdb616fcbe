// TGSample.swift -- Swift host side of the CUDA sampling engine (C ABI in
// include/tgsample.h, module CTGSample).
//
// What the reference's Swift host calls and what replaces it:
//   Serve.sampleToken(from:temperature:constraint:)      Serve.swift:1483-1506
//       -> ServeSampler.sampleToken(logits:request:constraint:uniform:)
//   request fields temperature / grammar / stop / stop_token_ids / max_tokens
//                                                        Serve.swift:758-763
//       -> SamplingRequest (adds top_k, top_p, min_p and the three penalties)
//   ServeConstraint.mask() / commit(tokenId:)            Serve.swift:1972-1978
//       -> GrammarConstraint (tg_grammar_*: a mask-table row instead of a
//          [Float] mask of the whole vocabulary per token)
//   SpeculativeDecode.step / stepStochastic              SpeculativeDecode.swift:41-210
//   MedusaVerify.step / EagleVerify.step (greedy)        MedusaHeads.swift:186-265,
//                                                        EagleDraft.swift:216-290
//       -> Sampler.verify (draft logits optional: greedy without a draft)
//
// Not compiled in this repository's build (no Swift toolchain on the build
// machine); the C ABI it calls is tested from C and Python.

import CTGSample
#if canImport(Glibc)
import Glibc
#elseif canImport(Darwin)
import Darwin
#endif

public struct TGError: Error, CustomStringConvertible {
    public let code: Int32
    public let message: String
    public var description: String { "tgsample error \(code): \(message)" }
}

@inline(__always)
func check(_ rc: Int32) throws {
    if rc != TG_OK { throw TGError(code: rc, message: String(cString: tg_last_error_string())) }
}

@inline(__always)
func checkGrammar(_ rc: Int32) throws {
    if rc != TG_OK { throw TGError(code: rc, message: String(cString: tg_grammar_last_error())) }
}

/// The sampling fields of a chat / completion request.  The first five are the
/// reference's (Serve.swift:758-763, same JSON names and defaults); the others
/// are this engine's additions, absent from the reference's requests.
public struct SamplingRequest {
    public var maxTokens: Int = 128
    public var temperature: Float = 0.0          // <= 0: greedy (Serve.swift:1495)
    public var stop: [String] = []
    public var stopTokenIds: [Int32] = []
    public var grammar: String? = nil            // JSON Schema text or the tool-tag GBNF
    public var topK: Int32 = 0                   // <= 0: off
    public var topP: Float = 1.0                 // >= 1: off
    public var minP: Float = 0.0                 // <= 0: off
    public var repetitionPenalty: Float = 1.0    // <= 1: off (ModelController.swift:268-284)
    public var presencePenalty: Float = 0.0
    public var frequencyPenalty: Float = 0.0

    public init() {}

    /// Reads the request JSON the way Serve.swift:758-763 reads its fields.
    public init(json: [String: Any]) {
        maxTokens = (json["max_tokens"] as? Int) ?? 128
        temperature = (json["temperature"] as? Double).map { Float($0) } ?? 0.0
        if let s = json["stop"] as? String { stop = [s] } else { stop = (json["stop"] as? [String]) ?? [] }
        stopTokenIds = ((json["stop_token_ids"] as? [Int]) ?? []).map { Int32($0) }
        if let g = json["grammar"] as? String { grammar = g }
        topK = Int32((json["top_k"] as? Int) ?? 0)
        topP = (json["top_p"] as? Double).map { Float($0) } ?? 1.0
        minP = (json["min_p"] as? Double).map { Float($0) } ?? 0.0
        repetitionPenalty = (json["repetition_penalty"] as? Double).map { Float($0) } ?? 1.0
        presencePenalty = (json["presence_penalty"] as? Double).map { Float($0) } ?? 0.0
        frequencyPenalty = (json["frequency_penalty"] as? Double).map { Float($0) } ?? 0.0
    }

    /// The per-row record tg_sample reads.
    public var rowParams: tg_row_params {
        tg_row_params(temperature: temperature, top_p: topP, min_p: minP,
                      repetition_penalty: repetitionPenalty, presence_penalty: presencePenalty,
                      frequency_penalty: frequencyPenalty, top_k: topK, flags: 0)
    }
}

/// One tg_sampler handle: one CUDA device, one stream at a time (the handle's
/// buffers are per handle; use one Sampler per stream).
public final class Sampler {
    let h: OpaquePointer
    public let vocab: Int32
    public let maxBatch: Int32

    public init(device: Int32 = 0, vocab: Int32, maxBatch: Int32) throws {
        var p: OpaquePointer? = nil
        try check(tg_sampler_create(device, vocab, maxBatch, &p))
        h = p!
        self.vocab = vocab
        self.maxBatch = maxBatch
    }

    deinit { tg_sampler_destroy(h) }

    /// Buffers for verification of up to maxK proposals and the vocab-sharded
    /// call over up to maxRanks ranks; call once before the decode loop.
    public func reserve(maxK: Int32, maxRanks: Int32 = 0) throws {
        try check(tg_sampler_reserve(h, maxK, maxRanks))
    }

    /// One row of host fp32 logits (the last position, as Serve.sampleToken gets
    /// them) through the host-buffer entry point.  `maskRow`: the grammar row
    /// (ceil(vocab/32) words) of the sequence's state, nil when unconstrained.
    public func sampleToken(logits: [Float], request: SamplingRequest, history: [Int32] = [],
                            maskRow: [UInt32]? = nil, uniform: Float) throws -> (token: Int32, prob: Float) {
        var params = request.rowParams
        var id: Int32 = -1, prob: Float = 0, u = uniform
        var hlen = Int32(history.count), sid: Int32 = 0
        let hist = history.isEmpty ? [Int32(0)] : history
        try logits.withUnsafeBufferPointer { lp in
            try hist.withUnsafeBufferPointer { hp in
                if let mask = maskRow {
                    try mask.withUnsafeBufferPointer { mp in
                        try check(tg_sample_host(h, lp.baseAddress, TG_DTYPE_F32, Int64(logits.count), 1,
                                                 &params, hp.baseAddress, &hlen, Int32(hist.count),
                                                 mp.baseAddress, 1, &sid, &u, &id, &prob))
                    }
                } else {
                    try check(tg_sample_host(h, lp.baseAddress, TG_DTYPE_F32, Int64(logits.count), 1,
                                             &params, hp.baseAddress, &hlen, Int32(hist.count),
                                             nil, 0, nil, &u, &id, &prob))
                }
            }
        }
        return (id, prob)
    }

    /// A batch on the device (logits stay where the model wrote them): device
    /// pointers, asynchronous on `stream` (a cudaStream_t, nil = default stream).
    public func sample(logits: UnsafeRawPointer, dtype: Int32, rowStride: Int64, batch: Int32,
                       params: UnsafePointer<tg_row_params>, history: UnsafePointer<Int32>?,
                       historyLen: UnsafePointer<Int32>?, historyStride: Int32,
                       maskTable: UnsafePointer<UInt32>?, numStates: Int32, stateId: UnsafePointer<Int32>?,
                       uniforms: UnsafePointer<Float>, outIds: UnsafeMutablePointer<Int32>,
                       outProbs: UnsafeMutablePointer<Float>? = nil,
                       stream: UnsafeMutableRawPointer? = nil) throws {
        try check(tg_sample(h, logits, dtype, rowStride, batch, params, history, historyLen, historyStride,
                            maskTable, numStates, stateId, uniforms, outIds, outProbs, stream))
    }

    /// Speculative verification of a batch (SpeculativeDecode.swift:41-210).
    /// Greedy rows (temperature <= 0) verify by argmax; with `draft` and
    /// `uAccept` nil every row must be greedy (Medusa / EAGLE heads have no draft
    /// distribution).  With `stateRows` the verification runs under the grammar.
    public func verify(target: UnsafeRawPointer, draft: UnsafeRawPointer?, dtype: Int32,
                       batch: Int32, k: Int32, draftIds: UnsafePointer<Int32>,
                       temperature: UnsafePointer<Float>, uAccept: UnsafePointer<Float>?,
                       uDraw: UnsafePointer<Float>, outIds: UnsafeMutablePointer<Int32>,
                       outCount: UnsafeMutablePointer<Int32>, maskTable: UnsafePointer<UInt32>? = nil,
                       numStates: Int32 = 0, stateRows: UnsafePointer<Int32>? = nil,
                       stream: UnsafeMutableRawPointer? = nil) throws {
        if let rows = stateRows, let table = maskTable {
            try check(tg_spec_verify_masked(h, target, draft, dtype, batch, k, draftIds, temperature,
                                            uAccept, uDraw, table, numStates, rows, outIds, outCount, stream))
        } else {
            try check(tg_spec_verify(h, target, draft, dtype, batch, k, draftIds, temperature,
                                     uAccept, uDraw, outIds, outCount, stream))
        }
    }

    /// Device status bits of the last completed call (see tgsample.h).
    public func deviceStatus() throws -> UInt32 {
        var bits: UInt32 = 0
        try check(tg_sampler_device_status(h, &bits))
        return bits
    }
}

/// A compiled grammar (JSON Schema or the tool-tag GBNF) over one tokenizer's
/// vocabulary; one per (grammar text, tokenizer), shared by every request.
public final class Grammar {
    let g: OpaquePointer
    public let vocab: Int32

    /// tokenBytes[i] = the bytes of token i (Serve.cachedTokenBytes); eosId -1
    /// gives the serve masker's rule (nothing allowed once the document is complete).
    public init(text: String, tokenBytes: [[UInt8]], eosId: Int32 = -1) throws {
        var flat: [UInt8] = []
        var offsets: [Int64] = [0]
        for t in tokenBytes {
            flat.append(contentsOf: t)
            offsets.append(Int64(flat.count))
        }
        if flat.isEmpty { flat = [0] }
        var p: OpaquePointer? = nil
        let utf8 = Array(text.utf8)
        try utf8.withUnsafeBufferPointer { tp in
            try tp.withMemoryRebound(to: CChar.self) { cp in
                try checkGrammar(tg_grammar_create(cp.baseAddress, Int64(utf8.count), Int32(tokenBytes.count),
                                                   flat, offsets, eosId, &p))
            }
        }
        g = p!
        vocab = Int32(tokenBytes.count)
    }

    deinit { tg_grammar_destroy(g) }

    /// The mask table (rows x ceil(vocab/32) words) to upload as tg_sample's
    /// mask_table; it grows when a state meets a new row.
    public func table() throws -> (words: UnsafePointer<UInt32>, rows: Int32) {
        var w: UnsafePointer<UInt32>? = nil
        var rows: Int32 = 0
        try checkGrammar(tg_grammar_table(g, &w, &rows))
        return (w!, rows)
    }
}

/// One sequence's automaton: the replacement of ServeConstraint
/// (Serve.swift:1945-1978).  Instead of a [Float] mask of the whole vocabulary
/// per token it hands out a row of the grammar's mask table.
public final class GrammarConstraint {
    let s: OpaquePointer
    public let grammar: Grammar

    public init(_ grammar: Grammar) throws {
        var p: OpaquePointer? = nil
        try checkGrammar(tg_grammar_state_create(grammar.g, &p))
        s = p!
        self.grammar = grammar
    }

    deinit { tg_grammar_state_destroy(s) }

    /// The state's row in the mask table (tg_sample's state_id); isNew when the
    /// row was just added (upload it before sampling).
    public func row() throws -> (row: Int32, isNew: Bool) {
        var r: Int32 = 0, n: Int32 = 0
        try checkGrammar(tg_grammar_state_row(s, &r, &n))
        return (r, n != 0)
    }

    /// The state's mask as words (bit i % 32 of word i / 32 = token i).
    public func maskWords() throws -> [UInt32] {
        var out = [UInt32](repeating: 0, count: Int((grammar.vocab + 31) / 32))
        try checkGrammar(tg_grammar_mask(s, &out))
        return out
    }

    /// ServeConstraint.commit(tokenId:): false leaves the state unchanged.
    @discardableResult
    public func commit(tokenId: Int32) throws -> Bool {
        var ok: Int32 = 0
        try checkGrammar(tg_grammar_commit(s, tokenId, &ok))
        return ok != 0
    }

    public func isComplete() throws -> Bool {
        var done: Int32 = 0
        try checkGrammar(tg_grammar_is_complete(s, &done))
        return done != 0
    }
}

/// The serve loop's sampling call with the reference's shape
/// (Serve.swift:1483-1506: token and the time spent in the constraint), over
/// this engine: the request's parameters, the constraint's mask row, the
/// row's recent tokens for the penalties, and a caller-drawn uniform (the
/// reference draws inside MLXRandom.categorical; here the draw is explicit so
/// it is reproducible).
public final class ServeSampler {
    public let sampler: Sampler

    public init(device: Int32 = 0, vocab: Int32) throws {
        sampler = try Sampler(device: device, vocab: vocab, maxBatch: 1)
    }

    public func sampleToken(logits: [Float], request: SamplingRequest, constraint: GrammarConstraint?,
                            recentTokens: [Int32] = [], uniform: Float) throws -> (token: Int, constraintMs: Double) {
        var mask: [UInt32]? = nil
        var constraintMs = 0.0
        if let c = constraint {
            let t0 = DispatchTimeShim.nowNs()
            mask = try c.maskWords()
            constraintMs = Double(DispatchTimeShim.nowNs() - t0) / 1e6
        }
        let (token, _) = try sampler.sampleToken(logits: logits, request: request, history: recentTokens,
                                                 maskRow: mask, uniform: uniform)
        if let c = constraint { try c.commit(tokenId: token) }
        return (Int(token), constraintMs)
    }
}

/// A monotonic nanosecond clock without Foundation.
enum DispatchTimeShim {
    static func nowNs() -> UInt64 {
        var ts = timespec()
        clock_gettime(CLOCK_MONOTONIC, &ts)
        return UInt64(ts.tv_sec) * 1_000_000_000 + UInt64(ts.tv_nsec)
    }
}
