"""Writes the golden fixtures of tests/golden from the reference itself.

Run in a container that has the reference tree (the argument, else $KRAFLA_REF,
else BASELINE.json's reference_path) and
the reference build of oracle/_ref (make -C oracle ref):

    python tests/golden/gen_golden.py [REFERENCE_ROOT [MODEL ...]]

Fixtures (all small; committed):
  models/*.mlb        models written by the reference's tools/gen_random.py
                      (the Makefile recipes of its e2e models)
  <model>.logits.npy  [16, vocab] logits of the reference's scalar build
                      (ml_forward of oracle/_ref/libkrafla_ref_scalar.so) for
                      TOKENS; the oracle must equal them bit for bit
  <model>.numpy.npy   the same from the reference's numpy forward
                      (tools/ref_forward.py), its float64 emulation
  quant.npz           float inputs and the reference's quantize_q8 /
                      quantize_q4 outputs (tools/mlb.py), f32 and f16 scales,
                      including zero, tiny, small and tie blocks
  writer_tiny.mlb     a model written by the reference's write_mlb from the
                      float weights of this repository's seeded generator
                      (kw_normal), for a byte-for-byte check of the C writer
"""
import ctypes as C
import os
import subprocess
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import oracle as _oracle  # noqa: E402
REF = sys.argv[1] if len(sys.argv) > 1 else _oracle.reference_root()
if not REF:
    sys.exit("gen_golden: the reference tree is not here (pass it, or set KRAFLA_REF)")
sys.path.insert(0, os.path.join(REF, "tools"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "isa-lm_b200"))
import mlb  # noqa: E402  (the reference's format module)
import ref_forward  # noqa: E402
import oracle  # noqa: E402
import krafla_b200  # noqa: E402

TOKENS = [1, 5, 9, 13, 17, 21, 25, 29, 33, 37, 41, 45, 49, 53, 57, 61]   # tests/test_e2e.sh:11

# name -> tools/gen_random.py arguments (reference Makefile:79-142 recipes, plus f16 and llama3 variants)
MODELS = {
    "rand_q8": ["--wtype", "q8"],
    "rand_q4": ["--wtype", "q4"],
    "mix_q4": ["--wtype", "q4", "--q8", "emb,v,o,down", "--seed", "4"],
    "mixf16_q4": ["--wtype", "q4", "--q8", "v,o,down", "--seed", "6", "--scales", "f16"],
    "bias_q4": ["--wtype", "q4", "--qkv-bias", "--seed", "7"],
    "llama3_q4": ["--wtype", "q4", "--rope-scaling", "32,1,4,8", "--seed", "9", "--scales", "f16"],
    "swa_q8": ["--wtype", "q8", "--sliding-window", "6", "--seed", "4"],
    "ctx_q4": ["--wtype", "q4", "--dim", "128", "--layers", "2", "--heads", "4", "--kv-heads", "2",
               "--hidden", "256", "--vocab", "96", "--max-seq", "160", "--seed", "11"],
    # the reference's feature models (Makefile:93-128)
    "qk_q4": ["--wtype", "q4", "--head-dim", "32", "--qk-norm", "--qkv-bias", "--seed", "4"],
    "lwin_q8": ["--wtype", "q8", "--layers", "4", "--sliding-window", "5", "--layer-pattern", "2",
                "--rope-local-theta", "100", "--scales", "f16", "--seed", "5"],
    "gemma_q4": ["--wtype", "q4", "--layers", "4", "--head-dim", "32", "--qk-norm", "--sliding-window", "5",
                 "--layer-pattern", "2", "--rope-local-theta", "100", "--gelu", "--post-norms", "--embed-scale", "8",
                 "--attn-scale", "0.2", "--scales", "f16", "--seed", "4"],
    "g2_q8": ["--wtype", "q8", "--layers", "4", "--sliding-window", "5", "--layer-pattern", "2", "--gelu",
              "--post-norms", "--embed-scale", "8", "--attn-scale", "0.25", "--attn-softcap", "2",
              "--final-softcap", "3", "--scales", "f16", "--seed", "4"],
    "yarn_q4": ["--wtype", "q4", "--rope-yarn", "4,8", "--seed", "4"],
}


def gen_models(only=None):
    os.makedirs(os.path.join(HERE, "models"), exist_ok=True)
    ref = oracle.RefBuild("scalar")
    for name, args in MODELS.items():
        if only and name not in only:
            continue
        path = os.path.join(HERE, "models", f"{name}.mlb")
        subprocess.run([sys.executable, os.path.join(REF, "tools", "gen_random.py"), "--out", path, *args], check=True)
        h = ref.open(path, 1, 0, False)
        cfg, t = mlb.read_mlb(path)
        vocab = cfg["vocab"]
        out = np.zeros((len(TOKENS), vocab), np.float32)
        for p, tok in enumerate(TOKENS):
            assert ref.L.ref_forward(h, tok, p, out[p].ctypes.data_as(C.c_void_p)) == 0
        ref.L.ref_close(h)
        np.save(os.path.join(HERE, f"{name}.logits.npy"), out)
        np.save(os.path.join(HERE, f"{name}.numpy.npy"), ref_forward.forward(cfg, t, TOKENS))
        print("wrote", name)


def gen_quant():
    rng = np.random.default_rng(20261201)
    xs = []
    for scale in (0.02, 1.0, 1e-7, 3.0):
        x = (rng.standard_normal(64 * 32) * scale).astype(np.float32)
        x[:32] = 0.0                                   # zero block
        x[32:64] = np.where(np.arange(32) % 2, 1e-37, -3e-37).astype(np.float32)   # 127/amax = inf
        x[64:96] *= np.float32(1e-4)
        x[96:128] = 0.0
        x[96], x[97:102] = 127.0, [0.5, -0.5, 1.5, 2.5, -2.5]   # tests/test_quant.c:47-60 ties
        x[128 + 3], x[128 + 9] = -5.0, 4.999                       # tests/test_quant.c:37-45 clamp
        xs.append(x)
    x = np.concatenate(xs)
    out = {"x": x}
    for f16 in (False, True):
        q8, d8 = mlb.quantize_q8(x, f16)
        q4, d4 = mlb.quantize_q4(x, None, f16)
        tag = "f16" if f16 else "f32"
        out[f"q8_{tag}"], out[f"d8_{tag}"] = q8, np.asarray(d8)
        out[f"q4_{tag}"], out[f"d4_{tag}"] = q4, np.asarray(d4)
    np.savez_compressed(os.path.join(HERE, "quant.npz"), **out)
    print("wrote quant.npz")


# the writer fixture: a tiny tied Q4 model with Q8 classes, qkv bias and llama3 RoPE scaling
WRITER_CFG = dict(dim=64, n_layers=2, n_heads=4, n_kv_heads=2, hidden_dim=128, vocab=96, max_seq=32,
                  rope_theta=500000.0, wtype="q4", q8=("v", "o", "down"), shared=1, qkv_bias=1,
                  rope_scaling=("llama3", 32.0, 1.0, 4.0, 8192), seed=3)


def normal(tid, n, sigma, seed):
    g = krafla_b200.gen()
    out = np.empty(n, np.float32)
    g.kw_normal(seed, tid, 0, n, sigma, out.ctypes.data_as(C.c_void_p))
    return out


def gen_writer():
    c = WRITER_CFG
    seed, dim, hid = c["seed"], c["dim"], c["hidden_dim"]
    hd = dim // c["n_heads"]
    qd, kvd = hd * c["n_heads"], hd * c["n_kv_heads"]
    mat = lambda tid, r, k: normal(tid, r * k, 0.02, seed).reshape(r, k)  # noqa: E731
    w = {"tok_emb": mat(1, c["vocab"], dim), "layers": []}
    for l in range(c["n_layers"]):
        b = 100 + 16 * l
        w["layers"].append({
            "attn_norm": np.ones(dim, np.float32), "wq": mat(b + 1, qd, dim), "wk": mat(b + 2, kvd, dim),
            "wv": mat(b + 3, kvd, dim), "wo": mat(b + 4, dim, qd), "bq": normal(b + 5, qd, 0.02, seed),
            "bk": normal(b + 6, kvd, 0.02, seed), "bv": normal(b + 7, kvd, 0.02, seed),
            "ffn_norm": np.ones(dim, np.float32), "w1": mat(b + 9, hid, dim), "w2": mat(b + 10, dim, hid),
            "w3": mat(b + 11, hid, dim)})
    w["final_norm"] = np.ones(dim, np.float32)
    cfg = dict(dim=dim, n_layers=c["n_layers"], n_heads=c["n_heads"], n_kv_heads=c["n_kv_heads"], hidden_dim=hid,
               vocab=c["vocab"], max_seq=c["max_seq"], rope_theta=c["rope_theta"], norm_eps=1e-5,
               shared_classifier=1, qkv_bias=1,
               rope_scaling={"type": "llama3", "factor": 32.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                             "original_max_position_embeddings": 8192})
    mlb.write_mlb(os.path.join(HERE, "writer_tiny.mlb"), cfg, w, "q4", list(c["q8"]), scales="f16")
    print("wrote writer_tiny.mlb")


if __name__ == "__main__":
    only = sys.argv[2:]   # model names: regenerate just those
    gen_models(only)
    if not only:
        gen_quant()
        gen_writer()
