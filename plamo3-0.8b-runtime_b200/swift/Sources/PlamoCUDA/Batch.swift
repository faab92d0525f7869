import CPlamo

/// Drop-in for the reference `Batch` (Sources/Plamo/Batch.swift:4-187): independent lanes that
/// share the runtime's weights, one weight pass per step. The reference CLI uses four lanes
/// (--batch4); the library takes 1...64.
public final class Batch {
    public let handle: OpaquePointer
    public let runtime: Runtime
    public let lanes: Int

    /// Batch.init(_:) — Batch.swift:33-78.
    public init(_ runtime: Runtime, lanes: Int = 4) throws {
        var h: OpaquePointer?
        try check(plamo_batch_open(runtime.handle, Int32(lanes), &h))
        guard let h else { throw Failure.message("plamo_batch_open returned no handle") }
        handle = h
        self.runtime = runtime
        self.lanes = lanes
    }

    deinit { plamo_batch_close(handle) }

    /// Batch.prefill(_:) — Batch.swift:80-106: prompt i to lane i; the lanes' greedy next ids.
    public func prefill(_ prompts: [[Int]]) throws -> [Int] {
        let arrays = prompts.map { $0.map { Int32(truncatingIfNeeded: $0) } }
        let lengths = arrays.map { Int32($0.count) }
        var next = [Int32](repeating: -1, count: max(1, arrays.count))
        // stable base addresses for the prompt arrays while the call runs
        let buffers = arrays.map { array -> UnsafeMutableBufferPointer<Int32> in
            let b = UnsafeMutableBufferPointer<Int32>.allocate(capacity: max(1, array.count))
            _ = b.initialize(from: array)
            return b
        }
        defer { buffers.forEach { $0.deallocate() } }
        var pointers: [UnsafePointer<Int32>?] = buffers.map { UnsafePointer($0.baseAddress) }
        try check(plamo_batch_prefill(handle, &pointers, lengths, Int32(arrays.count), &next))
        return next.prefix(arrays.count).map { Int($0) }
    }

    /// Batch.step(_:) — Batch.swift:109-179: nil marks an inactive lane.
    public func step(_ tokens: [Int?]) throws -> [Int] {
        let ids = tokens.map { $0.map { Int32(truncatingIfNeeded: $0) } ?? -1 }
        var next = [Int32](repeating: -1, count: max(1, ids.count))
        try check(plamo_batch_step(handle, ids, Int32(ids.count), &next))
        return next.prefix(ids.count).map { Int($0) }
    }

    /// Batch.reset() — Batch.swift:182.
    public func reset() { plamo_batch_reset(handle) }

    public var gpuSeconds: Double { plamo_batch_gpu_seconds(handle) }
}
