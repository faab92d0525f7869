"""TEST INFRASTRUCTURE ONLY: ctypes wrapper around the CPU restatement in plamo_oracle.cpp.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference arm import this
module, as the checker or the timed CPU baseline. It never backs the product path.

`OracleRuntime` / `OracleBatch` mirror the reference's `Runtime` (Sources/Plamo/Runtime.swift)
and `Batch` (Sources/Plamo/Batch.swift) call surfaces. Weights are read straight from the model
directory: `model.safetensors` by memmap, or with `packed=True` the `.p12` archive is decoded with
an independent numpy restatement of Kernels.metal:23-31 and checked bit-identical to the bf16
tensors (the reference's PackedTests invariant) before use.
"""
from __future__ import annotations

import ctypes
import json
import os
import struct
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "liboracle.so"

_u16p = ctypes.POINTER(ctypes.c_uint16)
_f32p = ctypes.POINTER(ctypes.c_float)
_i32p = ctypes.POINTER(ctypes.c_int32)


class _Config(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in
                ("d", "layers", "heads", "kv_heads", "ffn", "vocab", "window", "pattern", "context")]


class _Layer(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in
                ("pre_mixer", "post_mixer", "pre_mlp", "post_mlp", "qkv", "o", "q_norm", "k_norm", "gate_up", "down")]


def build() -> Path:
    """Compile the oracle library (make in oracle/)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = ctypes.CDLL(str(LIB_PATH))
        L.oracle_create.restype = ctypes.c_void_p
        L.oracle_create.argtypes = [ctypes.POINTER(_Config), ctypes.POINTER(_Layer), ctypes.c_void_p, ctypes.c_void_p,
                                    ctypes.c_void_p, _f32p, _f32p]
        L.oracle_destroy.argtypes = [ctypes.c_void_p]
        L.oracle_reset.argtypes = [ctypes.c_void_p]
        L.oracle_position.argtypes = [ctypes.c_void_p]
        L.oracle_forward.argtypes = [ctypes.c_void_p, _i32p, ctypes.c_int, ctypes.c_int, _i32p]
        L.oracle_prefill.argtypes = [ctypes.c_void_p, _i32p, ctypes.c_int, _i32p]
        L.oracle_logits.argtypes = [ctypes.c_void_p, ctypes.c_int, _f32p]
        L.oracle_logits_bits.argtypes = [ctypes.c_void_p, ctypes.c_int, _u16p]
        L.oracle_hidden.argtypes = [ctypes.c_void_p, _f32p]
        L.oracle_kv.argtypes = [ctypes.c_void_p, ctypes.c_int, _u16p, _u16p]
        L.oracle_last_error.restype = ctypes.c_char_p
        L.oracle_batch_create.restype = ctypes.c_void_p
        L.oracle_batch_create.argtypes = [ctypes.c_void_p, ctypes.c_int]
        L.oracle_batch_destroy.argtypes = [ctypes.c_void_p]
        L.oracle_batch_reset.argtypes = [ctypes.c_void_p]
        L.oracle_batch_prefill.argtypes = [ctypes.c_void_p, ctypes.POINTER(_i32p), _i32p, ctypes.c_int, _i32p]
        L.oracle_batch_step.argtypes = [ctypes.c_void_p, _i32p, ctypes.c_int, _i32p]
        L.oracle_batch_logits_bits.argtypes = [ctypes.c_void_p, ctypes.c_int, _u16p]
        L.oracle_batch_hidden.argtypes = [ctypes.c_void_p, ctypes.c_int, _f32p]
        L.oracle_batch_kv.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, _u16p, _u16p]
        L.oracle_linear.argtypes = [_u16p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
        L.oracle_norm.argtypes = [_u16p, _f32p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_float, _f32p, _u16p, _f32p]
        L.oracle_swiglu.argtypes = [_f32p, _f32p, ctypes.c_int, ctypes.c_int]
        L.oracle_argmax_bits.restype = ctypes.c_uint32
        L.oracle_argmax_bits.argtypes = [_u16p, ctypes.c_int]
        L.oracle_argmax_f32.restype = ctypes.c_uint32
        L.oracle_argmax_f32.argtypes = [_f32p, ctypes.c_int]
        L.oracle_rope_tables.argtypes = [_f32p, _f32p, ctypes.c_int, ctypes.c_int, _u16p, _u16p]
        L.oracle_attention.argtypes = [_u16p, _u16p, _f32p] + [ctypes.c_int] * 8 + [_f32p, ctypes.c_int, ctypes.c_int, _f32p]
        L.oracle_packed_decode.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, _u16p]
        L.oracle_exp.argtypes = [_f32p, _f32p, ctypes.c_longlong]
        L.oracle_set_threads.argtypes = [ctypes.c_int]
        L.oracle_threads.restype = ctypes.c_int
        _lib = L
    return _lib


def _p(a, t):
    return a.ctypes.data_as(t)


def set_threads(n: int):
    lib().oracle_set_threads(int(n))


def threads() -> int:
    return int(lib().oracle_threads())


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even exactly as Kernels.metal:6-9 (including its NaN/inf arithmetic)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return (((u + 0x7FFF + ((u >> 16) & 1)) >> 16) & 0xFFFF).astype(np.uint16)


# ---------------------------------------------------------------------------------------
# model directory reading (independent of the product package)

def _read_safetensors(path: Path):
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(n))
    mm = np.memmap(path, dtype=np.uint8, mode="r")
    start = 8 + n
    out = {}
    for name, info in header.items():
        if name == "__metadata__":
            continue
        assert info["dtype"] == "BF16", name
        b, e = info["data_offsets"]
        out[name] = mm[start + b:start + e].view(np.uint16).reshape(info["shape"])
    return out


def _decode_p12_tensor(manifest, payload, name):
    """Kernels.metal:23-31 (packed_bits) restated in numpy over whole tensors."""
    rec = manifest["tensors"][name]
    if "raw" in rec:
        b, e = rec["raw"]
        return np.asarray(payload[b:e]).view(np.uint16).reshape(rec["shape"])
    ob, oe = rec["offsets"]
    db, de = rec["data"]
    entries = np.asarray(payload[ob:oe]).view(np.uint32)
    data = np.asarray(payload[db:de])
    out = np.empty((len(entries), 128), dtype=np.uint16)
    tagv = entries & 63
    base = (entries & ~np.uint32(63)).astype(np.int64)
    packed = tagv != 0
    if packed.any():
        enc = data[base[packed][:, None] + np.arange(192)]
        sm = enc[:, :128].astype(np.uint32)
        i = np.arange(128)
        code = (enc[:, 128 + i // 2] >> ((i % 2) * 4)) & 15
        minimum = (tagv[packed] + 107).astype(np.uint32)[:, None]
        exponent = np.where(code == 15, 0, minimum + code)
        out[packed] = ((sm & 127) | ((sm & 128) << 8) | (exponent << 7)).astype(np.uint16)
    if (~packed).any():
        out[~packed] = data[base[~packed][:, None] + np.arange(256)].view(np.uint16).reshape(-1, 128)
    return out.reshape(rec["shape"])


class Model:
    """Weights + config of one model directory, as numpy uint16 views."""

    def __init__(self, directory, packed: bool = False):
        d = Path(directory)
        self.dir = d
        self.config = json.loads((d / "config.json").read_text())
        freqs = json.loads((d / "config-mlx.json").read_text())["plamo_rope_inv_freq"]
        self.inv_local = np.array(freqs["local"], dtype=np.float32)
        self.inv_full = np.array(freqs["full"], dtype=np.float32)
        self.tensors = _read_safetensors(d / "model.safetensors")
        if packed:
            with open(d / "model.p12", "rb") as f:
                count = struct.unpack("<Q", f.read(8))[0]
                manifest = json.loads(f.read(count))
            payload = np.memmap(d / "model.p12", dtype=np.uint8, mode="r", offset=count + 8)
            for name in manifest["tensors"]:
                restored = _decode_p12_tensor(manifest, payload, name)
                if not np.array_equal(restored, self.tensors[name]):
                    raise AssertionError(f"packed tensor {name} is not bit-identical to the bf16 source")
                self.tensors[name] = restored


class OracleRuntime:
    """CPU counterpart of Runtime (Runtime.swift:128-553)."""

    def __init__(self, directory, context: int, packed: bool = False, model: Model | None = None):
        self.model = model or Model(directory, packed)
        c = self.model.config
        self.cfg = _Config(c["hidden_size"], c["num_hidden_layers"], c["num_attention_heads"],
                           c["num_key_value_heads"], c["intermediate_size"], c["vocab_size"],
                           c["window_size"], c["sliding_window_pattern"], context)
        t = self.model.tensors
        self._keep = []
        layers = (_Layer * self.cfg.layers)()
        for i in range(self.cfg.layers):
            p = f"model.layers.layers.{i}."
            names = ["pre_mixer_norm", "post_mixer_norm", "pre_mlp_norm", "post_mlp_norm", "mixer.qkv_proj",
                     "mixer.o_proj", "mixer.q_norm", "mixer.k_norm", "mlp.gate_up_proj", "mlp.down_proj"]
            ptrs = []
            for n in names:
                a = np.ascontiguousarray(t[p + n + ".weight"])
                self._keep.append(a)
                ptrs.append(a.ctypes.data)
            layers[i] = _Layer(*ptrs)
        self._layers = layers
        emb = np.ascontiguousarray(t["model.embed_tokens.weight"])
        fn = np.ascontiguousarray(t["model.norm.weight"])
        lm = np.ascontiguousarray(t["lm_head.weight"])
        self._keep += [emb, fn, lm]
        self.vocab = self.cfg.vocab
        self.hidden = self.cfg.d
        self.context = context
        self.h = lib().oracle_create(ctypes.byref(self.cfg), layers, emb.ctypes.data, fn.ctypes.data, lm.ctypes.data,
                                     _p(self.model.inv_local, _f32p), _p(self.model.inv_full, _f32p))
        if not self.h:
            raise RuntimeError(lib().oracle_last_error().decode())

    def __del__(self):
        if getattr(self, "h", None):
            lib().oracle_destroy(self.h)
            self.h = None

    def _check(self, rc):
        if rc:
            raise RuntimeError(lib().oracle_last_error().decode())

    def reset(self):
        lib().oracle_reset(self.h)

    @property
    def position(self) -> int:
        return lib().oracle_position(self.h)

    def prefill(self, ids) -> int:
        a = np.ascontiguousarray(ids, dtype=np.int32)
        out = ctypes.c_int32(-1)
        self._check(lib().oracle_prefill(self.h, _p(a, _i32p), len(a), ctypes.byref(out)))
        return out.value

    def forward(self, ids, output: bool = True) -> int:
        a = np.ascontiguousarray(ids, dtype=np.int32)
        out = ctypes.c_int32(-1)
        self._check(lib().oracle_forward(self.h, _p(a, _i32p), len(a), int(output), ctypes.byref(out)))
        return out.value

    def logits(self, slot: int = 0) -> np.ndarray:
        out = np.empty(self.vocab, dtype=np.float32)
        self._check(lib().oracle_logits(self.h, slot, _p(out, _f32p)))
        return out

    def logits_bits(self, slot: int = 0) -> np.ndarray:
        out = np.empty(self.vocab, dtype=np.uint16)
        self._check(lib().oracle_logits_bits(self.h, slot, _p(out, _u16p)))
        return out

    def hidden_state(self) -> np.ndarray:
        out = np.empty(self.hidden, dtype=np.float32)
        self._check(lib().oracle_hidden(self.h, _p(out, _f32p)))
        return out

    def kv(self, layer: int):
        cap = self.context if layer % self.cfg.pattern == self.cfg.pattern - 1 else min(self.context, self.cfg.window + min(self.context, 16))
        n = cap * self.cfg.kv_heads * 128
        k = np.empty(n, dtype=np.uint16); v = np.empty(n, dtype=np.uint16)
        self._check(lib().oracle_kv(self.h, layer, _p(k, _u16p), _p(v, _u16p)))
        return k, v

    def generate(self, prompt, steps: int, forced=None):
        """Greedy (or teacher-forced) decode; returns (ids, per-step bf16 logits list)."""
        nxt = self.prefill(prompt)
        ids, logits = [nxt], [self.logits_bits()]
        for i in range(steps - 1):
            tok = forced[i] if forced is not None else nxt
            nxt = self.forward([tok])
            ids.append(nxt)
            logits.append(self.logits_bits())
        return ids, logits


class OracleBatch:
    """CPU counterpart of Batch (Batch.swift:4-187) with `lanes` lanes."""

    def __init__(self, runtime: OracleRuntime, lanes: int = 4):
        self.rt = runtime
        self.lanes = lanes
        self.h = lib().oracle_batch_create(runtime.h, lanes)
        if not self.h:
            raise RuntimeError(lib().oracle_last_error().decode())

    def __del__(self):
        if getattr(self, "h", None):
            lib().oracle_batch_destroy(self.h)
            self.h = None

    def prefill(self, prompts):
        arrs = [np.ascontiguousarray(p, dtype=np.int32) for p in prompts]
        ptrs = (_i32p * len(arrs))(*[_p(a, _i32p) for a in arrs])
        lens = np.array([len(a) for a in arrs], dtype=np.int32)
        out = np.empty(len(arrs), dtype=np.int32)
        self.rt._check(lib().oracle_batch_prefill(self.h, ptrs, _p(lens, _i32p), len(arrs), _p(out, _i32p)))
        self._n = len(arrs)
        return out.tolist()

    def step(self, tokens):
        a = np.array([-1 if t is None else t for t in tokens], dtype=np.int32)
        out = np.empty(len(a), dtype=np.int32)
        self.rt._check(lib().oracle_batch_step(self.h, _p(a, _i32p), len(a), _p(out, _i32p)))
        return out.tolist()

    def reset(self):
        lib().oracle_batch_reset(self.h)

    def logits_bits(self, lane: int) -> np.ndarray:
        out = np.empty(self.rt.vocab, dtype=np.uint16)
        lib().oracle_batch_logits_bits(self.h, lane, _p(out, _u16p))
        return out

    def hidden_state(self, lane: int) -> np.ndarray:
        out = np.empty(self.rt.hidden, dtype=np.float32)
        lib().oracle_batch_hidden(self.h, lane, _p(out, _f32p))
        return out


# ---------------------------------------------------------------------------------------
# noise floor of the restatement itself

def _reordered(fn, mode: str = "reverse"):
    """Runs fn with every global-layer attention row through 16-key split-K partitions and every
    projection sum either walked backwards ("reverse": the same arithmetic in another fp32 order)
    or summed exactly and rounded once ("exact": the correctly rounded dot product, which is what
    fp32 accumulation on the tensor cores approaches)."""
    L = lib()
    L.oracle_set_split_partition.argtypes = [ctypes.c_int]
    L.oracle_set_dot_reverse.argtypes = [ctypes.c_int]
    L.oracle_set_split_partition(16)
    L.oracle_set_dot_reverse(2 if mode == "exact" else 1)
    try:
        return fn()
    finally:
        L.oracle_set_split_partition(0)
        L.oracle_set_dot_reverse(0)


def noise_floor(directory, context: int, prompt, steps: int, model: Model | None = None,
                mode: str = "reverse") -> dict:
    """Teacher-forced logit differences between the restatement and its reordered twin.

    A model whose activations are rounded to bf16 after every op amplifies fp32 reordering into
    bf16 rounding flips; this measures how far two correct implementations drift on a given model,
    which sets the scale for comparing the CUDA path (which sums in yet another order)."""
    model = model or Model(directory)
    a = OracleRuntime(directory, context, model=model)
    b = OracleRuntime(directory, context, model=model)
    nxt = a.prefill(prompt)
    _reordered(lambda: b.prefill(prompt), mode)
    rmse, maxabs = [], []
    for step in range(steps + 1):
        e = a.logits() - b.logits()
        rmse.append(float(np.sqrt(np.mean(e * e))))
        maxabs.append(float(np.max(np.abs(e))))
        if step == steps:
            break
        tok = nxt
        nxt = a.forward([tok])
        _reordered(lambda: b.forward([tok]), mode)
    return dict(rmse=max(rmse), maxabs=max(maxabs), rmse_mean=float(np.mean(rmse)))


# ---------------------------------------------------------------------------------------
# kernel-level restatements

def linear(w: np.ndarray, x: np.ndarray, logits: bool = False) -> np.ndarray:
    w = np.ascontiguousarray(w, dtype=np.uint16)
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, K = x.shape
    M = w.shape[0]
    y = np.empty((rows, M), dtype=np.uint16 if logits else np.float32)
    lib().oracle_linear(_p(w, _u16p), _p(x, _f32p), rows, K, M, int(logits), y.ctypes.data)
    return y


def norm(w, x, offset, residual=None, next_w=None):
    w = np.ascontiguousarray(w, dtype=np.uint16)
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, n = x.shape
    y = np.empty_like(x)
    res = None if residual is None else np.ascontiguousarray(residual, dtype=np.float32).copy()
    nw = None if next_w is None else np.ascontiguousarray(next_w, dtype=np.uint16)
    ny = None if next_w is None else np.empty_like(x)
    lib().oracle_norm(_p(w, _u16p), _p(x, _f32p), _p(y, _f32p), rows, n, offset,
                      None if res is None else _p(res, _f32p), None if nw is None else _p(nw, _u16p),
                      None if ny is None else _p(ny, _f32p))
    return y, ny


def argmax_bits(v: np.ndarray) -> int:
    v = np.ascontiguousarray(v, dtype=np.uint16)
    return int(lib().oracle_argmax_bits(_p(v, _u16p), len(v)))


def argmax_f32(v: np.ndarray) -> int:
    v = np.ascontiguousarray(v, dtype=np.float32)
    return int(lib().oracle_argmax_f32(_p(v, _f32p), len(v)))


def rope_tables(inv_local, inv_full, local_rows: int, context: int):
    il = np.ascontiguousarray(inv_local, dtype=np.float32)
    ig = np.ascontiguousarray(inv_full, dtype=np.float32)
    lo = np.empty(local_rows * 128, dtype=np.uint16)
    gl = np.empty(context * 128, dtype=np.uint16)
    lib().oracle_rope_tables(_p(il, _f32p), _p(ig, _f32p), local_rows, context, _p(lo, _u16p), _p(gl, _u16p))
    return lo, gl


def attention(keys, values, q, heads, kv_heads, cap, first, count, begin, end, full, inv_local, local_rows, split=0):
    keys = np.ascontiguousarray(keys, dtype=np.uint16)
    values = np.ascontiguousarray(values, dtype=np.uint16)
    q = np.ascontiguousarray(q, dtype=np.float32)
    il = np.ascontiguousarray(inv_local, dtype=np.float32)
    out = np.empty(heads * 128, dtype=np.float32)
    lib().oracle_attention(_p(keys, _u16p), _p(values, _u16p), _p(q, _f32p), heads, kv_heads, cap, first, count,
                           begin, end, int(full), _p(il, _f32p), local_rows, split, _p(out, _f32p))
    return out


def exp(x: np.ndarray) -> np.ndarray:
    """The restatement's software exp (the same IEEE operation sequence as the CUDA path)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x)
    lib().oracle_exp(_p(x, _f32p), _p(y, _f32p), x.size)
    return y


def packed_decode(data: np.ndarray, entries: np.ndarray, count: int) -> np.ndarray:
    data = np.ascontiguousarray(data, dtype=np.uint8)
    entries = np.ascontiguousarray(entries, dtype=np.uint32)
    out = np.empty(count, dtype=np.uint16)
    lib().oracle_packed_decode(data.ctypes.data, entries.ctypes.data, count, _p(out, _u16p))
    return out


# ---------------------------------------------------------------------------------------
# decoding controls (Sampler.swift), restated for the device sampler's parity tests

def sampler_forbidden(history, n: int) -> set:
    """Sampler.forbidden (Sampler.swift:54-70): ids that would complete an n-gram whose first n-1
    tokens equal the history's last n-1 tokens."""
    if n <= 1 or len(history) < n:
        return set()
    span = n - 1
    last = len(history) - span
    out = set()
    for start in range(last):
        if all(history[start + o] == history[last + o] for o in range(span)):
            out.add(history[start + span])
    return out


def sampler_select(logits, history, penalty: float, no_repeat_ngram: int, frequency: float = 0.0,
                   presence: float = 0.0) -> int:
    """Sampler.select (Sampler.swift:9-31) in fp32: per history id (count c) the repetition penalty
    (x / p when x > 0, else x * p), minus presence, minus frequency * c; -inf for forbidden ids;
    then the first index whose value exceeds every earlier one, starting from -inf (0 if none)."""
    v = np.array(logits, dtype=np.float32).copy()
    V = len(v)
    p, fr, pr = np.float32(penalty), np.float32(frequency), np.float32(presence)
    if p != 1 or pr != 0 or fr != 0:
        counts = {}
        for i in history:
            if 0 <= i < V:
                counts[i] = counts.get(i, 0) + 1
        for i, c in counts.items():
            x = v[i]
            if p != 1:
                x = x / p if x > 0 else x * p
            if pr != 0:
                x = x - pr
            if fr != 0:
                x = x - fr * np.float32(c)
            v[i] = x
    if no_repeat_ngram > 1:
        for i in sampler_forbidden(list(history), no_repeat_ngram):
            if 0 <= i < V:
                v[i] = -np.inf
    with np.errstate(invalid="ignore"):
        ok = v > -np.inf
    if not ok.any():
        return 0
    best = v[ok].max()
    return int(np.flatnonzero(ok & (v == best))[0])


def sampler_repetition_period(tokens, repeats: int):
    """Sampler.repetitionPeriod (Sampler.swift:35-51): shortest period 1...32 whose block repeats
    max(repeats, ceil(24 / period)) times at the tail, else None."""
    if repeats < 2 or len(tokens) < repeats:
        return None
    for period in range(1, 33):
        count = max(repeats, (24 + period - 1) // period)
        span = period * count
        if len(tokens) < span:
            continue
        start = len(tokens) - span
        if all(tokens[start + o] == tokens[start + o % period] for o in range(span)):
            return period
    return None
