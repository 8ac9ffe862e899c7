"""Synthetic BASELINE models: their configurations, the files that hold them
and their headers, in plain Python.

Nothing here loads a library of this repository. Files are written by the
`mlbgen` command (isa-lm_b200/csrc/mlbgen_main.c over mlb_writer.c) in a
child process, and headers are read with struct at the offsets of the .mlb
header table (reference docs/file-format.md). bench.py's CPU reference arm
uses this module, so that its process maps only the reference's own build.

Seed-to-bytes recipe of a file: tensor t (ids: tok_emb 1, wcls 2, final_norm
3, layer l's tensors 100 + 16 l + k in file order) element i takes the
Box-Muller normal of two uniforms drawn by SplitMix64 from (seed, t, i), times
sigma; norm weights are 1.0; each matrix is then quantized by the reference's
writer rules (tools/mlb.py: Q8_0, or the fitted Q4_0 rule) with f16 scales.
The same seed gives the same bytes for any thread count.
"""
import os
import struct
import subprocess

_HERE = os.path.dirname(os.path.abspath(__file__))
MLBGEN = os.path.join(_HERE, "krafla_b200", "mlbgen")

Q8M = {"emb": 1, "cls": 2, "qk": 4, "v": 8, "o": 16, "up": 32, "down": 64}

# synthetic N(0, 0.02) weights, norms 1.0, f16 block scales.
CONFIGS = {
    "cfg0": dict(dim=288, n_layers=6, n_heads=6, n_kv_heads=6, hidden_dim=768, vocab=32000, max_seq=256,
                 rope_theta=10000.0, wtype="q8"),
    "cfg1": dict(dim=896, n_layers=24, n_heads=14, n_kv_heads=2, hidden_dim=4864, vocab=151936, max_seq=512,
                 rope_theta=1e6, wtype="q4", q8=("v", "o", "down"), shared=1, qkv_bias=1),
    "cfg2": dict(dim=2048, n_layers=16, n_heads=32, n_kv_heads=8, hidden_dim=8192, vocab=128256, max_seq=4096,
                 rope_theta=5e5, wtype="q4", q8=("v", "o", "down"), shared=1,
                 rope_scaling=("llama3", 32.0, 1.0, 4.0, 8192)),
    "cfg4": dict(dim=4096, n_layers=32, n_heads=32, n_kv_heads=8, hidden_dim=14336, vocab=128256, max_seq=8192,
                 rope_theta=5e5, wtype="q8"),
}


def write_model(path, dim, n_layers, n_heads, n_kv_heads, hidden_dim, vocab, max_seq, rope_theta=10000.0,
                norm_eps=1e-5, wtype="q8", q8=(), shared=0, qkv_bias=0, head_dim=0, rope_scaling=None,
                scale_f16=1, sigma=0.02, bias_sigma=0.02, seed=0, nthreads=None):
    """Writes a synthetic .mlb (seeded N(0, sigma) weights, the reference's
    quantization rules and file layout) with the mlbgen command."""
    if not os.path.exists(MLBGEN):
        raise RuntimeError(f"{MLBGEN} missing: build it (make -C isa-lm_b200/csrc)")
    a = dict(dim=dim, n_layers=n_layers, n_heads=n_heads, n_kv_heads=n_kv_heads, hidden_dim=hidden_dim,
             vocab=vocab, max_seq=max_seq, rope_theta=repr(float(rope_theta)), norm_eps=repr(float(norm_eps)),
             wtype=1 if wtype == "q8" else 2, shared=int(bool(shared)), qkv_bias=int(bool(qkv_bias)),
             head_dim=head_dim, scale_f16=int(bool(scale_f16)), q8_mask=sum(Q8M[k] for k in q8),
             sigma=repr(float(sigma)), bias_sigma=repr(float(bias_sigma)), seed=int(seed),
             nthreads=nthreads or os.cpu_count() or 1)
    if rope_scaling:
        kind = rope_scaling[0]
        a["rope_type"] = {"llama3": 1, "linear": 2}[kind]
        a["rope_factor"] = repr(float(rope_scaling[1]))
        if kind == "llama3":
            a["rope_lo"], a["rope_hi"] = repr(float(rope_scaling[2])), repr(float(rope_scaling[3]))
            a["rope_orig"] = int(rope_scaling[4])
    r = subprocess.run([MLBGEN, os.fspath(path)] + [f"{k}={v}" for k, v in a.items()], capture_output=True, text=True)
    if r.returncode:
        raise OSError(r.returncode, f"writing {path}: {r.stderr.strip()}")


def model_path(name, directory, seed=0, **overrides):
    """Where ensure_model keeps BASELINE config `name`."""
    tag = "" if not overrides else "_" + "_".join(f"{k}{v}" for k, v in sorted(overrides.items()))
    return os.path.join(directory, f"{name}{tag}_s{seed}.mlb")


def ensure_model(name, directory, seed=0, **overrides):
    """Path of BASELINE config `name` (CONFIGS) in `directory`, written once."""
    cfg = dict(CONFIGS[name], **overrides)
    path = model_path(name, directory, seed, **overrides)
    if not os.path.exists(path):
        os.makedirs(directory, exist_ok=True)
        tmp = path + f".tmp{os.getpid()}"
        write_model(tmp, seed=seed, **cfg)
        os.replace(tmp, path)
    return path


_HEADER_U32 = ("dim", "n_layers", "n_heads", "n_kv_heads", "hidden_dim", "vocab", "max_seq")


def read_header(path):
    """The shape fields of an .mlb header (offsets 8..35 and 44..51, 80),
    with head_dim, q_dim and kv_dim derived as the format specifies."""
    with open(path, "rb") as f:
        h = f.read(256)
    if len(h) < 256 or h[:4] != b"MLB1":
        raise ValueError(f"{path}: not an .mlb file")
    c = dict(zip(_HEADER_U32, struct.unpack_from("<7I", h, 8)))
    c["rope_theta"], c["norm_eps"] = struct.unpack_from("<2f", h, 36)
    c["wtype"], c["shared"] = struct.unpack_from("<2I", h, 44)
    c["q8_mask"], c["qkv_bias"], hd = struct.unpack_from("<3I", h, 72)
    c["head_dim"] = hd or c["dim"] // c["n_heads"]
    c["q_dim"], c["kv_dim"] = c["head_dim"] * c["n_heads"], c["head_dim"] * c["n_kv_heads"]
    (c["scale_f16"],) = struct.unpack_from("<I", h, 120)
    return c
