"""Host-side mirror of Krafla's model API (JonPark0/isa-lm) over the B200 build.

The reference's C API (model/mlb.h, model/transformer.h) maps one to one:

    ml_model_load  -> Model(path)                 kc_model_load
    ml_model_pack  -> Model.upload()              kc_model_upload (HBM, once)
    ml_state_init  -> State(model, nthreads, kv)  kc_state_init
    ml_prefill     -> State.prefill(...)          kc_prefill
    ml_state.batch -> State.set_batch(b)          kc_set_batch
    ml_forward     -> State.forward(token, pos)   kc_forward
    ml_state_free  -> State.free()                kc_state_free

plus State.generate_greedy (the ml_run -T 0 / ml_bench decode loop on the
device). Every call goes through the C ABI of include/krafla_cuda.h in
libkrafla_cuda.so; there is no other implementation behind it: when the
library or a B200 is missing the calls raise.

Status codes and their meaning are the reference's ml_status (core/ml.h:7-14).
"""
import ctypes as C
import os
import sys

import numpy as np

_PARENT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if _PARENT not in sys.path:
    sys.path.insert(0, _PARENT)
# the synthetic models (configs, files, headers) live in a module of their own
# that loads no library: bench.py's CPU arm uses it without this package
from krafla_models import CONFIGS, Q8M, ensure_model, model_path, read_header, write_model  # noqa: E402,F401

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libkrafla_cuda.so")
GEN_PATH = os.path.join(_HERE, "libkrafla_mlbgen.so")

OK, E_IO, E_FORMAT, E_SHAPE, E_NOMEM, E_ISA = range(6)
F32, Q8_0, Q4_0, F16 = 0, 1, 2, 3
TP_MAX, TP_HANDLE_BYTES = 8, 64          # KC_TP_MAX, KC_TP_HANDLE_BYTES of include/krafla_cuda.h
STATUS = {OK: "ok", E_IO: "i/o error", E_FORMAT: "bad file format", E_SHAPE: "bad tensor shape",
          E_NOMEM: "out of memory", E_ISA: "device lacks required architecture"}


class KraflaError(RuntimeError):
    """A non-zero status from the C ABI; .status holds the ml_status value."""

    def __init__(self, status, what=""):
        self.status = status
        msg = STATUS.get(status, f"status {status}")
        super().__init__(f"{what}: {msg}" + (f" ({what_detail()})" if what_detail() else ""))


_lib = None
_gen = None


def what_detail():
    return _lib.kc_last_error().decode() if _lib is not None else ""


class _Config(C.Structure):
    """kc_config: the reference's ml_config field order (model/mlb.h:9-32)."""
    _fields_ = [(n, C.c_int) for n in ("dim", "n_layers", "n_heads", "n_kv_heads", "hidden_dim", "vocab",
                                       "max_seq", "head_dim", "kv_dim", "q_dim")] + [
        ("rope_theta", C.c_float), ("norm_eps", C.c_float), ("wtype", C.c_int), ("q8_mask", C.c_uint),
        ("qkv_bias", C.c_int), ("qk_norm", C.c_int), ("sliding_window", C.c_int), ("layer_flags", C.c_int),
        ("rope_local_theta", C.c_float), ("act", C.c_int), ("post_norms", C.c_int), ("embed_scale", C.c_float),
        ("attn_scale", C.c_float), ("scale_f16", C.c_int), ("attn_softcap", C.c_float),
        ("final_softcap", C.c_float), ("rope_type", C.c_int), ("rope_orig_max_seq", C.c_int),
        ("rope_factor", C.c_float), ("rope_low_freq_factor", C.c_float), ("rope_high_freq_factor", C.c_float),
        ("rope_attn_factor", C.c_float)]


def lib():
    """The loaded libkrafla_cuda.so (raises when it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} missing: build it (python -c 'import __graft_entry__ as g; g.build()')")
        L = C.CDLL(LIB_PATH)
        P, I, F, S = C.c_void_p, C.c_int, C.c_float, C.c_size_t
        sig = {
            "kc_device_check": (I, []), "kc_status_str": (C.c_char_p, [I]), "kc_last_error": (C.c_char_p, []),
            "kc_model_load": (I, [C.POINTER(P), C.c_char_p]), "kc_model_upload": (I, [P]),
            "kc_model_config": (C.POINTER(_Config), [P]), "kc_model_device_bytes": (S, [P]),
            "kc_model_free": (None, [P]),
            "kc_state_init": (I, [C.POINTER(P), P, I, I]), "kc_prefill": (I, [P, P, I, I, P]),
            "kc_set_batch": (I, [P, I]), "kc_model_shard": (I, [P, I, I]), "kc_model_shard_info": (I, [P, P]),
            "kc_set_device": (I, [I]), "kc_tp_handle": (I, [P, P, S]), "kc_tp_connect": (I, [P, P]),
            "kc_sampler_init": (I, [C.POINTER(P), P, P]), "kc_sampler_accept": (I, [P, I]),
            "kc_sample": (I, [P, C.POINTER(I)]), "kc_generate_sampled": (I, [P, P, I, I, I, P]),
            "kc_sampler_rng": (I, [P, C.POINTER(C.c_uint64)]), "kc_sampler_free": (None, [P]),
            "kc_forward": (C.POINTER(F), [P, I, I]), "kc_generate_greedy": (I, [P, I, I, I, P]),
            "kc_state_free": (None, [P]),
            "kc_time_decode": (I, [P, I, I, I, I, C.POINTER(F)]),
            "kc_step_timeline": (I, [P, I, I, P, I, C.POINTER(I)]),
            "kc_step_trace": (I, [P, I, I, P, S, C.POINTER(I), C.POINTER(I)]),
            "kc_step_events": (I, [P, I, I, P, C.c_uint, C.POINTER(I)]),
            "kc_quantize_q8_dev": (I, [P, P, P, I, P]), "kc_rmsnorm_quantize_dev": (I, [P, P, P, P, P, I, F, P]),
            "kc_matvec_dev": (I, [P, I, I, P, P, I, I, P, P, P]),
            "kc_matvec_f32_noalloc": (I, [P, I, I, P, P, I, I, P, P]),
            "kc_matmul_dev": (I, [P, I, I, P, P, I, I, P, P, I, P]), "kc_block_sums_dev": (I, [P, I, P, I, I, P, P]),
            "kc_dev_alloc": (P, [S]), "kc_dev_free": (None, [P]), "kc_memcpy_htod": (I, [P, P, S]),
            "kc_memcpy_dtoh": (I, [P, P, S]), "kc_dev_sync": (I, []), "kc_debug_wait_limit": (I, [I]),
            "kc_debug_ffn_split": (I, [I]),
        }
        for name, (res, args) in sig.items():
            f = getattr(L, name)
            f.restype, f.argtypes = res, args
        _lib = L
    return _lib


def _check(st, what):
    if st != OK:
        raise KraflaError(st, what)


class _SamplerOpts(C.Structure):
    _fields_ = [("temperature", C.c_float), ("topp", C.c_float), ("topk", C.c_int), ("repeat_penalty", C.c_float),
                ("repeat_last_n", C.c_int), ("seed", C.c_uint64)]


class Sampler:
    """ml_sampler on the device for a State: kc_sampler_init / accept / kc_sample."""

    def __init__(self, state, temperature=0.0, topp=0.0, topk=0, repeat_penalty=1.0, repeat_last_n=0, seed=0):
        self.state = state
        self._h = C.c_void_p()
        o = _SamplerOpts(temperature, topp, topk, repeat_penalty, repeat_last_n, seed)
        _check(lib().kc_sampler_init(C.byref(self._h), state._h, C.byref(o)), "sampler init")

    def accept(self, token):
        _check(lib().kc_sampler_accept(self._h, int(token)), "sampler accept")

    def sample(self):
        """ml_sample on the state's last logits (on the device)."""
        t = C.c_int()
        _check(lib().kc_sample(self._h, C.byref(t)), "sample")
        return t.value

    @property
    def rng(self):
        r = C.c_uint64()
        lib().kc_sampler_rng(self._h, C.byref(r))
        return r.value

    def free(self):
        if self._h:
            lib().kc_sampler_free(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def set_device(device):
    """The calling thread's CUDA device for this library (one rank, one GPU)."""
    _check(lib().kc_set_device(int(device)), "set device")


def exchange_handles(handle, dist):
    """Every rank's tensor-parallel handle, in rank order, through an initialised
    torch.distributed process group (any backend: objects travel on the CPU)."""
    out = [None] * dist.get_world_size()
    dist.all_gather_object(out, bytes(handle))
    if any(not isinstance(h, bytes) or len(h) != TP_HANDLE_BYTES for h in out):
        raise KraflaError(E_SHAPE, "tp handles: a rank sent a malformed handle")
    return out


def device_check():
    """0 on a B200 (sm_100) this build runs on; raises otherwise."""
    _check(lib().kc_device_check(), "device check")


class Model:
    """ml_model_load + ml_model_pack: map and validate an .mlb, upload it to HBM."""

    def __init__(self, path, upload=True):
        self._h = C.c_void_p()
        _check(lib().kc_model_load(C.byref(self._h), os.fsencode(path)), f"load {path}")
        if upload:
            self.upload()

    def upload(self):
        _check(lib().kc_model_upload(self._h), "upload")

    def shard(self, rank, world):
        """Keep rank's tensor-parallel share of world (before upload)."""
        _check(lib().kc_model_shard(self._h, int(rank), int(world)), "shard")
        return self

    @property
    def shard_info(self):
        v = (C.c_int * 9)()
        _check(lib().kc_model_shard_info(self._h, v), "shard info")
        keys = ("rank", "world", "n_heads", "n_kv_heads", "q_dim", "kv_dim", "hidden_dim", "cls_row0", "cls_rows")
        return dict(zip(keys, list(v)))

    @property
    def config(self):
        c = lib().kc_model_config(self._h).contents
        return {n: getattr(c, n) for n, _ in c._fields_}

    @property
    def device_bytes(self):
        return lib().kc_model_device_bytes(self._h)

    def free(self):
        if self._h:
            lib().kc_model_free(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class State:
    """ml_state: decode state with its HBM KV cache (kv_type F32, F16 or Q8_0)."""

    def __init__(self, model, nthreads=1, kv_type=F32):
        self.model = model
        self.cfg = model.config
        self._h = C.c_void_p()
        _check(lib().kc_state_init(C.byref(self._h), model._h, nthreads, kv_type), "state init")

    def forward(self, token, pos):
        """Logits [vocab] for token at pos (a copy), as ml_forward; None when out of range."""
        p = lib().kc_forward(self._h, int(token), int(pos))
        if not p:
            err = what_detail()
            if err:
                raise KraflaError(E_IO, f"forward: {err}")
            return None
        return np.ctypeslib.as_array(p, shape=(self.cfg["vocab"],)).copy()

    def prefill(self, tokens, pos0=0, logits=False):
        """ml_prefill: runs the tokens at pos0..; returns [n, vocab] logits or None."""
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        out = np.empty((len(t), self.cfg["vocab"]), np.float32) if logits else None
        st = lib().kc_prefill(self._h, t.ctypes.data_as(C.c_void_p), len(t), int(pos0),
                              out.ctypes.data_as(C.c_void_p) if logits else None)
        _check(st, "prefill")
        return out

    def tp_handle(self):
        """This rank's exchange-buffer handle (bytes) for the other ranks."""
        buf = C.create_string_buffer(TP_HANDLE_BYTES)
        _check(lib().kc_tp_handle(self._h, buf, TP_HANDLE_BYTES), "tp handle")
        return buf.raw

    def tp_connect(self, handles):
        """Open every rank's exchange buffer (handles in rank order)."""
        blob = b"".join(bytes(h) for h in handles)
        _check(lib().kc_tp_connect(self._h, blob), "tp connect")
        return self

    def set_batch(self, batch):
        """ml_state.batch: prompt tokens per batched prefill step (1 = token by token)."""
        _check(lib().kc_set_batch(self._h, int(batch)), "set batch")
        return self

    def generate_sampled(self, sampler, token, pos, n):
        """n tokens from token at pos, each sampled on the device by `sampler`."""
        out = np.empty(n, np.int32)
        _check(lib().kc_generate_sampled(self._h, sampler._h, int(token), int(pos), int(n),
                                         out.ctypes.data_as(C.c_void_p)), "generate sampled")
        return out

    def generate_greedy(self, token, pos, n):
        """n greedy tokens from token at pos, the loop kept on the device."""
        out = np.empty(n, np.int32)
        _check(lib().kc_generate_greedy(self._h, int(token), int(pos), int(n), out.ctypes.data_as(C.c_void_p)),
               "generate")
        return out

    def time_decode(self, token, pos, warmup, steps):
        ms = C.c_float()
        _check(lib().kc_time_decode(self._h, int(token), int(pos), int(warmup), int(steps), C.byref(ms)),
               "time decode")
        return ms.value

    def step_timeline(self, token, pos):
        """Device clock (ns) at the start of one step and after each of its grid
        barriers: per layer Q/K/V, attention, O, gate/up, down; then the classifier."""
        t = np.zeros(4096, np.uint64)
        n = C.c_int()
        _check(lib().kc_step_timeline(self._h, int(token), int(pos), t.ctypes.data_as(C.c_void_p), 4096, C.byref(n)),
               "timeline")
        return t[:n.value].astype(np.int64)

    def step_trace(self, token, pos):
        """[phase, cta, 3] device clock (ns): activation prologue done, barrier arrival, release."""
        cap = (5 * self.cfg["n_layers"] + 1) * 1024 * 3
        t = np.zeros(cap, np.uint64)
        P, G = C.c_int(), C.c_int()
        _check(lib().kc_step_trace(self._h, int(token), int(pos), t.ctypes.data_as(C.c_void_p), cap, C.byref(P),
                                   C.byref(G)), "trace")
        return t[:P.value * G.value * 3].astype(np.int64).reshape(P.value, G.value, 3)

    def step_events(self, token, pos, cap=4096):
        """[cta, who, cap] event words of one step (clock << 8 | code); who 0 consumer, 1 producer."""
        G = C.c_int()
        out = np.zeros(1024 * 2 * cap, np.uint64)
        _check(lib().kc_step_events(self._h, int(token), int(pos), out.ctypes.data_as(C.c_void_p), cap, C.byref(G)),
               "events")
        return out[:G.value * 2 * cap].reshape(G.value, 2, cap)

    def free(self):
        if self._h:
            lib().kc_state_free(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


# ---------------------------------------------------------------- device arrays

class DevBuf:
    """A device allocation through the C ABI (for the kernel-level entry points)."""

    def __init__(self, nbytes):
        self.nbytes = int(nbytes)
        self.ptr = lib().kc_dev_alloc(max(1, self.nbytes))
        if not self.ptr:
            raise KraflaError(E_NOMEM, "device alloc")

    @classmethod
    def of(cls, arr, pad=0):
        a = np.ascontiguousarray(arr)
        b = cls(a.nbytes + pad)
        if a.nbytes:
            _check(lib().kc_memcpy_htod(b.ptr, a.ctypes.data_as(C.c_void_p), a.nbytes), "htod")
        return b

    def get(self, dtype, count):
        out = np.empty(count, dtype)
        if out.nbytes:
            _check(lib().kc_memcpy_dtoh(out.ctypes.data_as(C.c_void_p), self.ptr, out.nbytes), "dtoh")
        return out

    def __del__(self):
        try:
            if self.ptr:
                lib().kc_dev_free(self.ptr)
        except Exception:
            pass


def quantize_q8(x):
    """ml_k_quantize_q8 on the device: (int8 q [k], float d [k/32])."""
    x = np.ascontiguousarray(x, np.float32)
    k = x.size
    bx, bq, bd = DevBuf.of(x), DevBuf(k), DevBuf(4 * (k // 32))
    _check(lib().kc_quantize_q8_dev(bq.ptr, bd.ptr, bx.ptr, k, None), "quantize")
    _check(lib().kc_dev_sync(), "sync")
    return bq.get(np.int8, k), bd.get(np.float32, k // 32)


def rmsnorm_quantize(x, w, eps):
    """RMSNorm then quantize_q8 on the device: (q, d, normalized floats)."""
    x = np.ascontiguousarray(x, np.float32)
    n = x.size
    bx, bw, bq, bd, bn = DevBuf.of(x), DevBuf.of(np.asarray(w, np.float32)), DevBuf(n), DevBuf(4 * (n // 32)), DevBuf(4 * n)
    _check(lib().kc_rmsnorm_quantize_dev(bq.ptr, bd.ptr, bn.ptr, bx.ptr, bw.ptr, n, C.c_float(eps), None), "rmsnorm")
    _check(lib().kc_dev_sync(), "sync")
    return bq.get(np.int8, n), bd.get(np.float32, n // 32), bn.get(np.float32, n)


def matvec(wtype, wq, wd, rows, cols, xq, xd):
    """ml_k_matvec_q8/q4 over all rows on the device. wd: float32 or float16 scales."""
    wd = np.ascontiguousarray(wd)
    d16 = int(wd.dtype == np.float16)
    bw, bd = DevBuf.of(wq), DevBuf.of(wd, pad=16)   # scale rows are read in 16-byte aligned spans
    bxq, bxd, by = DevBuf.of(np.asarray(xq, np.int8)), DevBuf.of(np.asarray(xd, np.float32)), DevBuf(4 * rows)
    _check(lib().kc_matvec_dev(by.ptr, wtype, d16, bw.ptr, bd.ptr, rows, cols, bxq.ptr, bxd.ptr, None), "matvec")
    _check(lib().kc_dev_sync(), "sync")
    return by.get(np.float32, rows)


def matmul(wtype, wq, wd, rows, cols, xq, xd):
    """ml_matmul on the device for n quantized rows xq [n, cols], xd [n, cols/32]: y [n, rows]."""
    wd = np.ascontiguousarray(wd)
    d16 = int(wd.dtype == np.float16)
    xq = np.ascontiguousarray(xq, np.int8)
    n = xq.shape[0]
    bw, bd = DevBuf.of(wq), DevBuf.of(wd, pad=16)
    bxq, bxd, by = DevBuf.of(xq), DevBuf.of(np.ascontiguousarray(xd, np.float32)), DevBuf(4 * rows * n)
    _check(lib().kc_matmul_dev(by.ptr, wtype, d16, bw.ptr, bd.ptr, rows, cols, bxq.ptr, bxd.ptr, n, None), "matmul")
    _check(lib().kc_dev_sync(), "sync")
    return by.get(np.float32, rows * n).reshape(n, rows)


def block_sums(wtype, wq, rows, cols, xq):
    """int32 [rows, cols/32] block dot products on the device."""
    bw, bx, bs = DevBuf.of(wq), DevBuf.of(np.asarray(xq, np.int8)), DevBuf(4 * rows * (cols // 32))
    _check(lib().kc_block_sums_dev(bs.ptr, wtype, bw.ptr, rows, cols, bx.ptr, None), "block sums")
    _check(lib().kc_dev_sync(), "sync")
    return bs.get(np.int32, rows * (cols // 32)).reshape(rows, cols // 32)


# ---------------------------------------------------------------- model writer

def gen():
    """The model writer's library (its quantizers and generator, for tests)."""
    global _gen
    if _gen is None:
        if not os.path.exists(GEN_PATH):
            raise RuntimeError(f"{GEN_PATH} missing: build it first")
        g = C.CDLL(GEN_PATH)
        g.kw_quantize.restype = C.c_int
        g.kw_quantize.argtypes = [C.c_int, C.c_int, C.c_void_p, C.c_long, C.c_void_p, C.c_void_p]
        g.kw_normal.restype = None
        g.kw_normal.argtypes = [C.c_uint64, C.c_uint64, C.c_uint64, C.c_long, C.c_double, C.c_void_p]
        _gen = g
    return _gen
