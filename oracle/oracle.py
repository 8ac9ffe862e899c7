"""TEST INFRASTRUCTURE ONLY — ctypes access to the CPU oracle (liboracle.so,
the C restatement of the reference's scalar token loop) and to the
reference's own build (oracle/_ref/libkrafla_ref_<isa>.so, compiled from the
reference sources by oracle/Makefile).

Only tests/, __graft_entry__.smoke() and bench.py's CPU baseline legs may use
this module; the CUDA product never imports it.
"""
import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_DIR = os.path.join(HERE, "_ref")
P, I, F = C.c_void_p, C.c_int, C.c_float

_orc = None


def reference_root():
    """The reference source tree: $KRAFLA_REF, else the `reference_path` of the
    repository's BASELINE.json; None when neither names a directory here (as
    on a machine without the reference, where the prebuilt oracle/_ref is used)."""
    root = os.environ.get("KRAFLA_REF")
    if not root:
        try:
            import json
            with open(os.path.join(os.path.dirname(HERE), "BASELINE.json")) as f:
                root = json.load(f).get("reference_path")
        except (OSError, ValueError):
            root = None
    return root if root and os.path.isdir(root) else None


def build(ref_root=None):
    """Builds liboracle.so, and oracle/_ref when the reference tree is present."""
    subprocess.run(["make", "-s", "-C", HERE, "liboracle.so"], check=True)
    ref_root = ref_root or reference_root()
    if ref_root:
        subprocess.run(["make", "-s", "-C", HERE, "ref", f"REF={ref_root}"], check=True)


def orc():
    global _orc
    if _orc is None:
        if not os.path.exists(ORACLE_SO):
            build()
        L = C.CDLL(ORACLE_SO)
        sig = {
            "orc_quantize_q8": (None, [P, P, P, I]), "orc_quantize_row": (None, [P, P, P, I]),
            "orc_matvec": (None, [P, I, P, P, I, I, P, P, I, I]), "orc_block_sums": (None, [P, I, P, I, I, P]),
            "orc_rmsnorm": (None, [P, P, P, I, F]), "orc_softmax": (None, [P, I]),
            "orc_rope": (None, [P, P, P, P, I, I, I]), "orc_silu_mul": (None, [P, P, I]),
            "orc_f32_to_f16": (C.c_uint16, [F]), "orc_f16_to_f32": (F, [C.c_uint16]),
            "orc_model_load": (I, [C.POINTER(P), C.c_char_p]), "orc_model_free": (None, [P]),
            "orc_model_config": (None, [P, P]), "orc_state_new": (I, [C.POINTER(P), P, I, I]),
            "orc_state_free": (None, [P]), "orc_forward": (I, [P, I, I, P]), "orc_prefill": (I, [P, P, I, I, P]),
            "orc_state_x": (C.POINTER(F), [P]),
            "orc_sampler_new": (I, [C.POINTER(P), I, P]), "orc_sampler_free": (None, [P]),
            "orc_sampler_accept": (None, [P, I]), "orc_sampler_rng": (C.c_uint64, [P]),
            "orc_sample": (I, [P, P, C.POINTER(F)]),
        }
        for name, (res, args) in sig.items():
            f = getattr(L, name)
            f.restype, f.argtypes = res, args
        _orc = L
    return _orc


class SamplerOpts(C.Structure):
    """ml_sampler_opts (model/sampler.h), field for field."""
    _fields_ = [("temperature", C.c_float), ("topp", C.c_float), ("topk", C.c_int), ("repeat_penalty", C.c_float),
                ("repeat_last_n", C.c_int), ("seed", C.c_uint64)]


def sampler_opts(temperature=0.0, topp=0.0, topk=0, repeat_penalty=1.0, repeat_last_n=0, seed=0):
    return SamplerOpts(temperature, topp, topk, repeat_penalty, repeat_last_n, seed)


class OracleSampler:
    """The oracle's restatement of the reference sampler: sample() returns the
    token and the draw's distance from the nearest token boundary (relative)."""

    def __init__(self, vocab, opts):
        self.h = C.c_void_p()
        if orc().orc_sampler_new(C.byref(self.h), vocab, C.byref(opts)):
            raise MemoryError("oracle sampler")
        self.vocab = vocab

    def accept(self, token):
        orc().orc_sampler_accept(self.h, int(token))

    def sample(self, logits):
        lg = np.array(logits, np.float32, copy=True)
        m = C.c_float()
        tok = orc().orc_sample(self.h, _ptr(lg), C.byref(m))
        return int(tok), float(m.value)

    @property
    def rng(self):
        return int(orc().orc_sampler_rng(self.h))

    def close(self):
        if self.h:
            orc().orc_sampler_free(self.h)
            self.h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _ptr(a):
    return a.ctypes.data_as(C.c_void_p)


def quantize_q8(x):
    x = np.ascontiguousarray(x, np.float32)
    q, d = np.empty(x.size, np.int8), np.empty(x.size // 32, np.float32)
    orc().orc_quantize_q8(_ptr(q), _ptr(d), _ptr(x), x.size)
    return q, d


def matvec(wtype, wq, wd, rows, cols, xq, xd):
    """Scalar matvec of the reference; wd: float32 scales [rows, cols/32]."""
    y = np.empty(rows, np.float32)
    wq, wd = np.ascontiguousarray(wq), np.ascontiguousarray(wd, np.float32)
    xq, xd = np.ascontiguousarray(xq, np.int8), np.ascontiguousarray(xd, np.float32)
    orc().orc_matvec(_ptr(y), wtype, _ptr(wq), _ptr(wd), rows, cols, _ptr(xq), _ptr(xd), 0, rows)
    return y


def block_sums(wtype, wq, rows, cols, xq):
    s = np.empty((rows, cols // 32), np.int32)
    wq, xq = np.ascontiguousarray(wq), np.ascontiguousarray(xq, np.int8)
    orc().orc_block_sums(_ptr(s), wtype, _ptr(wq), rows, cols, _ptr(xq))
    return s


def rmsnorm(x, w, eps):
    x, w = np.ascontiguousarray(x, np.float32), np.ascontiguousarray(w, np.float32)
    o = np.empty_like(x)
    orc().orc_rmsnorm(_ptr(o), _ptr(x), _ptr(w), x.size, eps)
    return o


CONFIG_FIELDS = ("dim", "n_layers", "n_heads", "n_kv_heads", "hidden_dim", "vocab", "max_seq", "head_dim", "kv_dim",
                 "q_dim", "wtype", "q8_mask", "qkv_bias", "qk_norm", "sliding_window", "act", "post_norms",
                 "scale_f16", "shared", "rope_type")


class OracleModel:
    """The oracle's decoder over one .mlb: forward / prefill with scalar semantics."""

    def __init__(self, path, kv_type=0, nthreads=None):
        self.m, self.s = C.c_void_p(), C.c_void_p()
        st = orc().orc_model_load(C.byref(self.m), os.fsencode(path))
        if st:
            raise RuntimeError(f"oracle load {path}: status {st}")
        f = (C.c_int * 20)()
        orc().orc_model_config(self.m, f)
        self.cfg = dict(zip(CONFIG_FIELDS, list(f)))
        st = orc().orc_state_new(C.byref(self.s), self.m, kv_type, nthreads or os.cpu_count() or 1)
        if st:
            raise RuntimeError(f"oracle state: status {st}")

    def forward(self, token, pos, logits=True):
        out = np.empty(self.cfg["vocab"], np.float32) if logits else None
        st = orc().orc_forward(self.s, int(token), int(pos), _ptr(out) if logits else None)
        if st:
            return None
        return out

    def prefill(self, tokens, pos0=0, logits=True):
        t = np.ascontiguousarray(tokens, np.int32)
        out = np.empty((len(t), self.cfg["vocab"]), np.float32) if logits else None
        st = orc().orc_prefill(self.s, _ptr(t), len(t), int(pos0), _ptr(out) if logits else None)
        if st:
            raise RuntimeError(f"oracle prefill: status {st}")
        return out

    def close(self):
        if self.s:
            orc().orc_state_free(self.s)
            self.s = C.c_void_p()
        if self.m:
            orc().orc_model_free(self.m)
            self.m = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ---------------------------------------------------------------- the reference build

def cpu_flags():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("flags"):
                    return set(line.split(":", 1)[1].split())
    except OSError:
        pass
    return set()


def best_ref_isa():
    """The reference's best build for this host: avx512vnni, else avx2, else scalar
    (the flags of tests/test_all.sh:16-25 in the reference)."""
    fl = cpu_flags()
    if {"avx512f", "avx512bw", "avx512_vnni"} <= fl:
        return "avx512vnni"
    if {"avx2", "fma", "f16c"} <= fl:
        return "avx2"
    return "scalar"


class RefBuild:
    """One of oracle/_ref/libkrafla_ref_<isa>.so (the unmodified reference library)."""

    def __init__(self, isa=None):
        self.isa = isa or best_ref_isa()
        path = os.path.join(REF_DIR, f"libkrafla_ref_{self.isa}.so")
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        L = C.CDLL(path)
        sig = {
            "ref_isa_name": (C.c_char_p, []), "ref_isa_ok": (I, []), "ref_open": (I, [P, I, I, I, C.POINTER(P)]),
            "ref_close": (None, [P]), "ref_forward": (I, [P, I, I, P]), "ref_prefill": (I, [P, P, I, I, P]),
            "ref_decode_greedy": (C.c_double, [P, I, I, I, P]), "ref_time_prefill": (C.c_double, [P, P, I, I]),
            "ref_threads": (I, [P]), "ref_set_batch": (None, [P, I]),
            "ref_quantize_q8": (None, [P, P, P, I]), "ref_quantize_q8_scalar": (None, [P, P, P, I]),
            "ref_matvec_scalar": (None, [P, I, P, P, I, I, P, P, I, I]),
            "ref_sample_seq": (I, [P, I, P, I, P, I, P, C.POINTER(C.c_uint64)]),
        }
        for name, (res, args) in sig.items():
            f = getattr(L, name)
            f.restype, f.argtypes = res, args
        self.L = L
        if L.ref_isa_ok() != 0:
            raise RuntimeError(f"this CPU cannot run the reference's {self.isa} build")

    def open(self, path, nthreads=1, kv_type=0, pack=True):
        h = C.c_void_p()
        st = self.L.ref_open(os.fsencode(path), nthreads, kv_type, int(pack), C.byref(h))
        if st:
            raise RuntimeError(f"reference ml_model_load/ml_state_init {path}: status {st}")
        return h

    def sample_seq(self, opts, vocab, context, logits):
        """The reference's ml_sampler over rows of logits (each choice accepted):
        (tokens, final rng state)."""
        lg = np.array(logits, np.float32, copy=True).reshape(-1, vocab)
        ctx = np.ascontiguousarray(context, np.int32)
        out = np.zeros(lg.shape[0], np.int32)
        rng = C.c_uint64()
        st = self.L.ref_sample_seq(C.byref(opts), vocab, _ptr(ctx), len(ctx), _ptr(lg), lg.shape[0], _ptr(out),
                                   C.byref(rng))
        if st:
            raise RuntimeError(f"reference sampler: status {st}")
        return out, int(rng.value)

