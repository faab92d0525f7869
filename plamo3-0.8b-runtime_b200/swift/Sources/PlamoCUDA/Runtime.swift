import CPlamo

/// Drop-in for the reference `Runtime` (Sources/Plamo/Runtime.swift:128-553) on a CUDA device:
/// the same members the engine calls (Main.swift, OrderedOutput.swift, BatchDecode.swift), each a
/// thin call into libplamo_cuda. Every call is synchronous, like the reference's
/// waitUntilCompleted; a handle is used from one thread at a time.
public final class Runtime {
    public let handle: OpaquePointer
    public let context: Int

    /// Runtime.init(directory:context:packed:) — Runtime.swift:164-286. `device` picks the CUDA
    /// device (the data-parallel launcher gives each process its own).
    public init(directory: String, context: Int, packed: Bool = false, device: Int = 0) throws {
        var h: OpaquePointer?
        try check(plamo_open(directory, Int32(context), packed ? 1 : 0, Int32(device), &h))
        guard let h else { throw Failure.message("plamo_open returned no handle") }
        handle = h
        self.context = context
    }

    deinit { plamo_close(handle) }

    /// Runtime.prefill(_:) — Runtime.swift:469-483.
    public func prefill(_ tokens: [Int]) throws -> Int {
        let ids = tokens.map { Int32(truncatingIfNeeded: $0) }
        var next: Int32 = -1
        try check(plamo_prefill(handle, ids, Int32(ids.count), &next))
        return Int(next)
    }

    /// Runtime.forward(_:output:) — Runtime.swift:321-467 (1...16 tokens at the current position).
    public func forward(_ tokens: [Int], output: Bool = true) throws -> Int {
        let ids = tokens.map { Int32(truncatingIfNeeded: $0) }
        var next: Int32 = -1
        try check(plamo_forward(handle, ids, Int32(ids.count), output ? 1 : 0, &next))
        return Int(next)
    }

    /// Runtime.reset() — Runtime.swift:319.
    public func reset() { plamo_reset(handle) }

    /// Runtime.logitValues(slot:) — Runtime.swift:540-545: bf16 logits widened to Float.
    public func logitValues(slot: Int = 0) -> [Float] {
        var values = [Float](repeating: 0, count: vocabulary)
        logits(into: &values, slot: slot)
        return values
    }

    /// Runtime.logits(into:slot:) — Runtime.swift:547-552; reuses `values`.
    public func logits(into values: inout [Float], slot: Int = 0) {
        if values.count != vocabulary { values = [Float](repeating: 0, count: vocabulary) }
        let status = values.withUnsafeMutableBufferPointer { plamo_logits(handle, Int32(slot), $0.baseAddress) }
        precondition(status == 0, String(cString: plamo_last_error()))
    }

    /// Sampler.select (Sampler.swift:9-31) on the device over slot 0's logits: only the history
    /// of generated ids travels, not the 107,520 logits.
    public func select(history: [Int], repetitionPenalty: Float, noRepeatNGram: Int, frequencyPenalty: Float,
                       presencePenalty: Float = 0) throws -> Int {
        let ids = history.map { Int32(truncatingIfNeeded: $0) }
        var out: Int32 = 0
        try check(plamo_select(handle, ids, Int32(ids.count), repetitionPenalty, Int32(noRepeatNGram),
                               frequencyPenalty, presencePenalty, &out))
        return Int(out)
    }

    public var position: Int { Int(plamo_position(handle)) }
    public var gpuSeconds: Double { plamo_gpu_seconds(handle) }
    /// Runtime.peakMetalBytes: the device bytes the runtime allocated.
    public var peakMetalBytes: Int { Int(plamo_device_bytes(handle)) }
    /// Weights.gpuBytes.
    public var weightBytes: Int { Int(plamo_weight_bytes(handle)) }
    public var deviceName: String { String(cString: plamo_device_name(handle)) }

    public var vocabulary: Int {
        var dims = [Int32](repeating: 0, count: 10)
        _ = plamo_dims(handle, &dims)
        return Int(dims[6])
    }
}
