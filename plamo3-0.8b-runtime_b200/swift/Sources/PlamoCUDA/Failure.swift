import CPlamo

/// The reference's error type (thrown as `Failure.message(...)` throughout Sources/Plamo): the
/// library's status codes become this error, carrying plamo_last_error()'s text, which uses the
/// reference's own messages ("Invalid tokens or context exhausted", "Input exceeds context", ...).
public enum Failure: Error, CustomStringConvertible {
    case message(String)
    public var description: String {
        switch self { case .message(let text): return text }
    }
}

@inline(__always) func check(_ status: Int32) throws {
    if status != 0 { throw Failure.message(String(cString: plamo_last_error())) }
}
