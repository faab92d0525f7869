"""Python mirror of the reference's `Runtime` / `Batch` interface over the C ABI (include/plamo.h).

    Runtime(directory, context, packed)      Runtime.init          Sources/Plamo/Runtime.swift:164
    .prefill(ids) -> next id                 Runtime.prefill       Runtime.swift:469-483
    .forward(ids, output=True) -> next id    Runtime.forward       Runtime.swift:321-467
    .logits(slot=0) -> float32[vocab]        Runtime.logits(into:) Runtime.swift:540-552
    .reset() / .position / .gpu_seconds      Runtime.swift:319, :154-155
    Batch(runtime, lanes=4)                  Batch.init            Sources/Plamo/Batch.swift:33-78
    .prefill(prompts) / .step(tokens)        Batch.swift:80-179    (None marks an inactive lane)
    .generate(prompts, limits)               Batch.generate + decodeBatch, BatchDecode.swift:8-47

Every call goes through libplamo_cuda.so; there is no CPU fallback. Importing this module without
the built library (or without a CUDA device at open time) raises.
"""
from __future__ import annotations

import atexit
import ctypes
import weakref
from pathlib import Path

import numpy as np

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libplamo_cuda.so"

_i32p = ctypes.POINTER(ctypes.c_int32)
_f32p = ctypes.POINTER(ctypes.c_float)
_u16p = ctypes.POINTER(ctypes.c_uint16)
_vp = ctypes.c_void_p


class PlamoError(RuntimeError):
    pass


_lib = None

# Open handles, closed batches-first at interpreter exit (before the CUDA runtime tears down), so
# finalizers never run in an unsafe order.
_open_batches = weakref.WeakSet()
_open_runtimes = weakref.WeakSet()


@atexit.register
def _close_all():
    for b in list(_open_batches):
        b.close()
    for r in list(_open_runtimes):
        r.close()


def library() -> ctypes.CDLL:
    """Loads libplamo_cuda.so (built by build.py). Fails loudly when it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise PlamoError(f"{LIB_PATH} is missing: run plamo3-0.8b-runtime_b200/build.py (there is no CPU fallback)")
    L = ctypes.CDLL(str(LIB_PATH))
    sig = {
        "plamo_open": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.POINTER(_vp)]),
        "plamo_open_broadcast": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, _vp,
                                                ctypes.c_int, ctypes.c_int, ctypes.POINTER(_vp)]),
        "plamo_nccl_unique_id": (ctypes.c_int, [_vp]),
        "plamo_broadcast_seconds": (ctypes.c_double, [_vp]),
        "plamo_close": (None, [_vp]),
        "plamo_prefill": (ctypes.c_int, [_vp, _i32p, ctypes.c_int, _i32p]),
        "plamo_forward": (ctypes.c_int, [_vp, _i32p, ctypes.c_int, ctypes.c_int, _i32p]),
        "plamo_logits": (ctypes.c_int, [_vp, ctypes.c_int, _f32p]),
        "plamo_hidden": (ctypes.c_int, [_vp, _f32p]),
        "plamo_reset": (None, [_vp]),
        "plamo_position": (ctypes.c_int, [_vp]),
        "plamo_gpu_seconds": (ctypes.c_double, [_vp]),
        "plamo_weight_bytes": (ctypes.c_size_t, [_vp]),
        "plamo_device_bytes": (ctypes.c_size_t, [_vp]),
        "plamo_device_name": (ctypes.c_char_p, [_vp]),
        "plamo_dims": (ctypes.c_int, [_vp, _i32p]),
        "plamo_batch_open": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.POINTER(_vp)]),
        "plamo_batch_prefill": (ctypes.c_int, [_vp, ctypes.POINTER(_i32p), _i32p, ctypes.c_int, _i32p]),
        "plamo_batch_step": (ctypes.c_int, [_vp, _i32p, ctypes.c_int, _i32p]),
        "plamo_batch_logits": (ctypes.c_int, [_vp, ctypes.c_int, _f32p]),
        "plamo_batch_hidden": (ctypes.c_int, [_vp, ctypes.c_int, _f32p]),
        "plamo_batch_reset": (None, [_vp]),
        "plamo_batch_gpu_seconds": (ctypes.c_double, [_vp]),
        "plamo_batch_close": (None, [_vp]),
        "plamo_batch_generate": (ctypes.c_int, [_vp, ctypes.POINTER(_i32p), _i32p, _i32p, ctypes.c_int, ctypes.c_int,
                                                _i32p, ctypes.c_int, _i32p, _i32p, _i32p]),
        "plamo_debug_kv": (ctypes.c_int, [_vp, ctypes.c_int, _u16p, _u16p]),
        "plamo_batch_debug_kv": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int, _u16p, _u16p]),
        "plamo_decode_chain": (ctypes.c_int, [_vp, ctypes.c_int, _i32p]),
        "plamo_step_launches": (ctypes.c_int, [_vp]),
        "plamo_profile_decode": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.POINTER(ctypes.c_double), _i32p]),
        "plamo_persistent_decode": (ctypes.c_int, [_vp]),
        "plamo_debug_wait_timeout": (ctypes.c_int, [_vp, ctypes.c_ulonglong]),
        "plamo_debug_nccl_init": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int, ctypes.c_longlong]),
        "plamo_trace_decode": (ctypes.c_int, [_vp, _vp, ctypes.c_size_t, _i32p]),
        "plamo_set_tensor_gemm": (ctypes.c_int, [_vp, ctypes.c_int]),
        "plamo_select": (ctypes.c_int, [_vp, _i32p, ctypes.c_int, ctypes.c_float, ctypes.c_int, ctypes.c_float,
                                        ctypes.c_float, _i32p]),
        "plamo_repetition_period": (ctypes.c_int, [_i32p, ctypes.c_int, ctypes.c_int]),
        "plamo_pack_p12": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_char_p, ctypes.POINTER(ctypes.c_uint64)]),
        "plamo_p12_chain_valid": (ctypes.c_int, [_vp, ctypes.c_size_t, ctypes.c_size_t]),
        "plamo_pack_blocks": (ctypes.c_int, [_vp, ctypes.c_size_t, _vp, ctypes.c_size_t, _vp,
                                             ctypes.POINTER(ctypes.c_size_t)]),
        "plamo_last_error": (ctypes.c_char_p, []),
        # kernel-level entry points (include/plamo_kernels.h)
        "plamo_k_linear": (ctypes.c_int, [_vp, _vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, _vp, _vp, _vp]),
        "plamo_k_linear_tc": (ctypes.c_int, [_vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, _vp, _vp,
                                             ctypes.c_int, _vp, ctypes.c_size_t, _vp]),
        "plamo_k_select": (ctypes.c_int, [_vp, ctypes.c_int, _vp, ctypes.c_int, ctypes.c_float, ctypes.c_int,
                                          ctypes.c_float, ctypes.c_float, _vp, _vp, _vp, _vp]),
        "plamo_k_argmax_keys": (ctypes.c_int, [_vp, ctypes.c_int, _vp, _vp]),
        "plamo_k_norm": (ctypes.c_int, [_vp, _vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_int, _vp, _vp, _vp]),
        "plamo_k_argmax": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int, _vp, _vp, _vp]),
        "plamo_k_packed_decode": (ctypes.c_int, [_vp, _vp, ctypes.c_longlong, _vp, _vp]),
        "plamo_k_attention": (ctypes.c_int, [_vp, _vp, _vp] + [ctypes.c_int] * 8 + [_vp, ctypes.c_int, _vp, _vp]),
        "plamo_k_attention_static": (ctypes.c_int, [_vp, _vp, _vp] + [ctypes.c_int] * 8 + [_vp, ctypes.c_int, _vp, _vp]),
        "plamo_k_attention_rows": (ctypes.c_int, [_vp, _vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, _vp, ctypes.c_int,
                                                  ctypes.c_int, _vp, ctypes.c_int, ctypes.c_int, _vp, _vp, ctypes.c_size_t,
                                                  _vp]),
        "plamo_k_exp": (ctypes.c_int, [_vp, _vp, ctypes.c_longlong, _vp]),
    }
    for name, (res, args) in sig.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    _lib = L
    return L


def _check(rc: int):
    if rc:
        raise PlamoError(library().plamo_last_error().decode())


def _ids(a):
    arr = np.ascontiguousarray(a, dtype=np.int32)
    return arr, arr.ctypes.data_as(_i32p)


class Runtime:
    """One model resident on one GPU (the reference's `Runtime`)."""

    def __init__(self, directory, context: int, packed: bool = False, device: int = 0, _handle=None):
        L = library()
        self._h = _vp()
        if _handle is not None:
            self._h = _handle
        else:
            _check(L.plamo_open(str(directory).encode(), int(context), int(bool(packed)), int(device), ctypes.byref(self._h)))
        _open_runtimes.add(self)
        dims = np.zeros(10, dtype=np.int32)
        _check(L.plamo_dims(self._h, dims.ctypes.data_as(_i32p)))
        (self.hidden_size, self.layers, self.heads, self.kv_heads, self.head_dim, self.ffn, self.vocab,
         self.window, self.pattern, self.context) = [int(v) for v in dims]

    @classmethod
    def broadcast(cls, directory, context: int, packed: bool, device: int, nccl_id: bytes, rank: int, world: int):
        """Data-parallel open: rank 0 reads the weights, every rank receives them by ncclBroadcast."""
        L = library()
        h = _vp()
        buf = ctypes.create_string_buffer(bytes(nccl_id), 128)
        _check(L.plamo_open_broadcast(str(directory).encode(), int(context), int(bool(packed)), int(device), buf,
                                      int(rank), int(world), ctypes.byref(h)))
        return cls(directory, context, packed, device, _handle=h)

    @staticmethod
    def nccl_unique_id() -> bytes:
        buf = ctypes.create_string_buffer(128)
        _check(library().plamo_nccl_unique_id(buf))
        return buf.raw

    def close(self):
        if self._h:
            library().plamo_close(self._h)
            self._h = _vp()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def prefill(self, ids) -> int:
        arr, p = _ids(ids)
        out = ctypes.c_int32(-1)
        _check(library().plamo_prefill(self._h, p, len(arr), ctypes.byref(out)))
        return out.value

    def forward(self, ids, output: bool = True) -> int:
        arr, p = _ids(ids)
        out = ctypes.c_int32(-1)
        _check(library().plamo_forward(self._h, p, len(arr), int(bool(output)), ctypes.byref(out)))
        return out.value

    def decode_chain(self, steps: int) -> list:
        out = np.empty(steps, dtype=np.int32)
        _check(library().plamo_decode_chain(self._h, int(steps), out.ctypes.data_as(_i32p)))
        return out.tolist()

    def step_launches(self) -> int:
        n = library().plamo_step_launches(self._h)
        if n < 0:
            _check(1)
        return n

    def profile_decode(self, steps: int):
        """Per-kernel-class device ms and launch counts over `steps` decode steps."""
        ms = (ctypes.c_double * 6)()
        n = np.zeros(6, dtype=np.int32)
        _check(library().plamo_profile_decode(self._h, int(steps), ms, n.ctypes.data_as(_i32p)))
        names = ["gemv", "qkv", "attention", "norm", "argmax", "persistent"]
        return {k: dict(ms=float(ms[i]), launches=int(n[i])) for i, k in enumerate(names) if n[i]}

    def trace_decode(self):
        """One decode step of the persistent kernel with its device timeline. Returns (phases,
        detail): phases is [CTAs, phases + 1, 3] nanoseconds relative to the earliest step begin
        (per phase [wait begin, work begin, work end]; the last record [step begin, head epilogue,
        step end]); detail is [CTAs, D] stamps inside the CTA's first layer-0 attention split
        (same origin; negative where unused)."""
        shape = np.zeros(4, dtype=np.int32)
        cap = 148 * 512 * 3
        while True:
            buf = np.zeros(cap, dtype=np.uint64)
            rc = library().plamo_trace_decode(self._h, buf.ctypes.data_as(ctypes.c_void_p), cap, shape.ctypes.data_as(_i32p))
            need = int(shape[0]) * ((int(shape[1]) + 1) * int(shape[2]) + int(shape[3]))
            if rc != 0 and need > cap:
                cap = need
                continue
            _check(rc)
            break
        G, P, S, D = (int(x) for x in shape)
        t = buf[: G * (P + 1) * S].reshape(G, P + 1, S).astype(np.int64)
        det = buf[G * (P + 1) * S: need].reshape(G, D).astype(np.int64)
        origin = t[:, -1, 0].min()
        return t - origin, np.where(det > 0, det - origin, -1)

    def select(self, history, penalty: float = 1.0, no_repeat_ngram: int = 0, frequency: float = 0.0,
               presence: float = 0.0) -> int:
        """Sampler.select (Sampler.swift:9-31) on the device over the current logits (slot 0)."""
        arr, ptr = _ids(history)
        out = ctypes.c_int32(0)
        _check(library().plamo_select(self._h, ptr, len(arr), float(penalty), int(no_repeat_ngram), float(frequency),
                                      float(presence), ctypes.byref(out)))
        return out.value

    def set_tensor_gemm(self, enable=True):
        """Tensor mode: True (or 3) puts the projections over >= 16 rows (prefill, batched steps) on
        the tcgen05 GEMM and the attention of calls over >= 16 rows on tcgen05 MMAs; 1 selects the
        projections only, 2 the attention only. Results within the accumulation-order tolerance of
        the default path, not bit for bit."""
        mode = 3 if enable is True else int(enable)
        _check(library().plamo_set_tensor_gemm(self._h, mode))

    @property
    def persistent(self) -> bool:
        return bool(library().plamo_persistent_decode(self._h))

    def debug_wait_timeout(self, limit_ns: int = 20_000):
        """Runs the persistent kernel's bounded poll on a device word nothing sets, with a short
        limit: raises PlamoError with the timed-out decode step's message; the runtime stays usable."""
        _check(library().plamo_debug_wait_timeout(self._h, int(limit_ns)))

    def logits(self, slot: int = 0) -> np.ndarray:
        out = np.empty(self.vocab, dtype=np.float32)
        _check(library().plamo_logits(self._h, int(slot), out.ctypes.data_as(_f32p)))
        return out

    logit_values = logits

    def hidden(self) -> np.ndarray:
        out = np.empty(self.hidden_size, dtype=np.float32)
        _check(library().plamo_hidden(self._h, out.ctypes.data_as(_f32p)))
        return out

    def reset(self):
        library().plamo_reset(self._h)

    def debug_kv(self, layer: int):
        cap = self.context if layer % self.pattern == self.pattern - 1 else min(self.context, self.window + min(self.context, 16))
        n = cap * self.kv_heads * 128
        k = np.empty(n, dtype=np.uint16); v = np.empty(n, dtype=np.uint16)
        _check(library().plamo_debug_kv(self._h, layer, k.ctypes.data_as(_u16p), v.ctypes.data_as(_u16p)))
        return k, v

    @property
    def position(self) -> int:
        return library().plamo_position(self._h)

    @property
    def gpu_seconds(self) -> float:
        return library().plamo_gpu_seconds(self._h)

    @property
    def weight_bytes(self) -> int:
        return library().plamo_weight_bytes(self._h)

    @property
    def device_bytes(self) -> int:
        return library().plamo_device_bytes(self._h)

    @property
    def device_name(self) -> str:
        return library().plamo_device_name(self._h).decode()

    @property
    def broadcast_seconds(self) -> float:
        return library().plamo_broadcast_seconds(self._h)


class Batch:
    """Independent sequences decoded together on one GPU (the reference's `Batch`)."""

    def __init__(self, runtime: Runtime, lanes: int = 4):
        self.runtime = runtime
        self.lanes = lanes
        self._h = _vp()
        _check(library().plamo_batch_open(runtime._h, int(lanes), ctypes.byref(self._h)))
        _open_batches.add(self)

    def close(self):
        # plamo_close already released the batches of a closed runtime
        if self._h and self.runtime._h:
            library().plamo_batch_close(self._h)
        self._h = _vp()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def prefill(self, prompts) -> list:
        arrs = [np.ascontiguousarray(p, dtype=np.int32) for p in prompts]
        ptrs = (_i32p * len(arrs))(*[a.ctypes.data_as(_i32p) for a in arrs])
        lens = np.array([len(a) for a in arrs], dtype=np.int32)
        out = np.empty(len(arrs), dtype=np.int32)
        _check(library().plamo_batch_prefill(self._h, ptrs, lens.ctypes.data_as(_i32p), len(arrs), out.ctypes.data_as(_i32p)))
        return out.tolist()

    def step(self, tokens) -> list:
        arr = np.array([-1 if t is None else t for t in tokens], dtype=np.int32)
        out = np.empty(len(arr), dtype=np.int32)
        _check(library().plamo_batch_step(self._h, arr.ctypes.data_as(_i32p), len(arr), out.ctypes.data_as(_i32p)))
        return out.tolist()

    def logits(self, lane: int) -> np.ndarray:
        out = np.empty(self.runtime.vocab, dtype=np.float32)
        _check(library().plamo_batch_logits(self._h, int(lane), out.ctypes.data_as(_f32p)))
        return out

    def hidden(self, lane: int) -> np.ndarray:
        out = np.empty(self.runtime.hidden_size, dtype=np.float32)
        _check(library().plamo_batch_hidden(self._h, int(lane), out.ctypes.data_as(_f32p)))
        return out

    def debug_kv(self, layer: int, lane: int):
        rt = self.runtime
        cap = rt.context if layer % rt.pattern == rt.pattern - 1 else min(rt.context, rt.window + min(rt.context, 16))
        n = cap * rt.kv_heads * 128
        k = np.empty(n, dtype=np.uint16); v = np.empty(n, dtype=np.uint16)
        _check(library().plamo_batch_debug_kv(self._h, layer, lane, k.ctypes.data_as(_u16p), v.ctypes.data_as(_u16p)))
        return k, v

    def reset(self):
        library().plamo_batch_reset(self._h)

    @property
    def gpu_seconds(self) -> float:
        return library().plamo_batch_gpu_seconds(self._h)

    def generate(self, prompts, limits, stop_on_truncation: bool = False):
        """Batch.generate / decodeBatch: list of (ids, reason) with reason "stop" or "length"."""
        n = len(prompts)
        arrs = [np.ascontiguousarray(p, dtype=np.int32) for p in prompts]
        ptrs = (_i32p * n)(*[a.ctypes.data_as(_i32p) for a in arrs])
        lens = np.array([len(a) for a in arrs], dtype=np.int32)
        lim = np.ascontiguousarray(limits, dtype=np.int32)
        stride = max(1, int(lim.max()) if n else 1)
        ids = np.zeros((n, stride), dtype=np.int32)
        out_lens = np.zeros(n, dtype=np.int32)
        reasons = np.zeros(n, dtype=np.int32)
        count = ctypes.c_int32(0)
        _check(library().plamo_batch_generate(self._h, ptrs, lens.ctypes.data_as(_i32p), lim.ctypes.data_as(_i32p), n,
                                              int(bool(stop_on_truncation)), ids.ctypes.data_as(_i32p), stride,
                                              out_lens.ctypes.data_as(_i32p), reasons.ctypes.data_as(_i32p),
                                              ctypes.byref(count)))
        return [(ids[i, :out_lens[i]].tolist(), "stop" if reasons[i] == 0 else "length") for i in range(count.value)]


def repetition_period(tokens, repeats: int):
    """Sampler.repetitionPeriod (Sampler.swift:35-51): the period, or None."""
    arr, ptr = _ids(tokens)
    p = library().plamo_repetition_period(ptr, len(arr), int(repeats))
    return p or None


def debug_nccl_init(nccl_id: bytes, rank: int, world: int, limit_ms: int) -> None:
    """The communicator setup of Runtime.broadcast alone, bounded by limit_ms (failure tests)."""
    buf = ctypes.create_string_buffer(bytes(nccl_id), 128)
    _check(library().plamo_debug_nccl_init(buf, int(rank), int(world), int(limit_ms)))


def pack_p12(model_dir, source_sha256: str | None = None) -> dict:
    """Writes model_dir/model.p12 with the library's C++ packer (pack_weights.py's archive bytes)."""
    stats = (ctypes.c_uint64 * 5)()
    _check(library().plamo_pack_p12(str(model_dir).encode(), source_sha256.encode() if source_sha256 else None, stats))
    keys = ("original_linear_bytes", "packed_linear_bytes", "archive_bytes", "compressed_blocks", "blocks")
    return dict(zip(keys, (int(v) for v in stats)))


def p12_chain_valid(entries, data_bytes: int) -> bool:
    """The loader's block-table check (Packed.swift:63-89) for one tensor."""
    e = np.ascontiguousarray(entries, dtype=np.uint32)
    return bool(library().plamo_p12_chain_valid(e.ctypes.data if e.size else None, e.size, int(data_bytes)))


def pack_blocks(values):
    """C++ block codec: (data uint8, tagged entries uint32) for a flat uint16 array."""
    v = np.ascontiguousarray(values, dtype=np.uint16).reshape(-1)
    data = np.empty(2 * v.size, dtype=np.uint8)
    entries = np.empty(v.size // 128, dtype=np.uint32)
    used = ctypes.c_size_t(0)
    _check(library().plamo_pack_blocks(v.ctypes.data, v.size, data.ctypes.data, data.size, entries.ctypes.data,
                                       ctypes.byref(used)))
    return data[: used.value], entries


def decode_batch(batch: Batch, prompts, limits, stop_on_truncation: bool = False):
    """Free-function form of BatchDecode.swift:41-47 (Batch.generate)."""
    return batch.generate(prompts, limits, stop_on_truncation)


# ----------------------------------------------------------------------------------------------
# kernel-level entry points on device pointers (include/plamo_kernels.h); pointers are ints
# (e.g. torch.Tensor.data_ptr()), stream an int cudaStream_t (0 = default stream).

def k_linear(w, offsets, x, rows, K, M, mode, y, keys=0, stream=0):
    _check(library().plamo_k_linear(w, offsets or None, x, rows, K, M, mode, y, keys or None, stream or None))


def k_linear_tc(w, x, rows, K, M, mode, y, keys=0, splits=0, workspace=0, workspace_floats=0, stream=0):
    _check(library().plamo_k_linear_tc(w, x, rows, K, M, mode, y, keys or None, int(splits), workspace or None,
                                       int(workspace_floats), stream or None))


def k_select(logits, V, history, n, penalty, no_repeat_ngram, frequency, presence, counts, flags, key_out, stream=0):
    _check(library().plamo_k_select(logits, V, history or None, n, float(penalty), int(no_repeat_ngram),
                                    float(frequency), float(presence), counts, flags, key_out, stream or None))


def select_key_to_id(key: int) -> int:
    """The id a plamo_k_select key stands for (0 when no value was above -inf)."""
    return 0 if key == 0 else 0xFFFFFFFF - (key & 0xFFFFFFFF)


def k_argmax_keys(keys, rows, out, stream=0):
    _check(library().plamo_k_argmax_keys(keys, rows, out, stream or None))


def k_norm(w, src, x, rows, n, offset, residual, next_w=0, next_out=0, stream=0):
    _check(library().plamo_k_norm(w, src, x, rows, n, float(offset), int(residual), next_w or None, next_out or None,
                                  stream or None))


def k_argmax(logits, rows, n, scratch, out, stream=0):
    _check(library().plamo_k_argmax(logits, rows, n, scratch, out, stream or None))


def k_packed_decode(data, entries, count, out, stream=0):
    _check(library().plamo_k_packed_decode(data, entries, int(count), out, stream or None))


def k_attention(q, keys, values, heads, kv_heads, cap, first, count, begin, end, full, rope_local, splits, out, stream=0):
    _check(library().plamo_k_attention(q, keys, values, heads, kv_heads, cap, first, count, begin, end, int(full),
                                       rope_local or None, splits, out, stream or None))


def k_attention_static(q, keys, values, heads, kv_heads, cap, first, count, begin, end, full, rope_local, splits, out,
                       stream=0):
    """plamo_k_attention on a fixed device scratch array (no device allocation; asynchronous)."""
    _check(library().plamo_k_attention_static(q, keys, values, heads, kv_heads, cap, first, count, begin, end, int(full),
                                              rope_local or None, splits, out, stream or None))


def k_attention_rows(q, keys, values, heads, kv_heads, cap, geo, rows, full, rope_local, splits, tensor, out,
                     workspace, workspace_bytes, stream=0):
    """plamo_k_attention_rows: multi-row (prefill) attention, CUDA-core or tensor-core kernel."""
    _check(library().plamo_k_attention_rows(q, keys, values, heads, kv_heads, cap, geo, rows, int(full),
                                            rope_local or None, splits, int(tensor), out, workspace,
                                            int(workspace_bytes), stream or None))


def k_exp(x, y, n, stream=0):
    _check(library().plamo_k_exp(x, y, int(n), stream or None))
