"""Benchmark of the B200 token loop (BASELINE metric: batch-1 decode tok/s and
% of HBM roofline; prefill tok/s; at 1/2/4/8 B200), one JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config cfg2] [--ctx 1024] [--tp-config cfg4] [--tp-ctx 2048]

N = 1 (one process): BASELINE config 2, the Llama-3.2-1B shape (Q4_0 with
v/o/down Q8_0, f16 scales, tied, llama3 RoPE), synthetic seeded weights;
batch-1 greedy decode at KV context --ctx (the prompt is prefilled first, then
W untimed and K timed decode steps). Weights (871 MB) are larger than the
126 MB L2, so every step streams them from HBM (no flush needed).

  value  decode tok/s: K tokens / the CUDA-event time of the K steps (one
         launch of the persistent step kernel; inputs in HBM)
  e2e    the same through the drop-in API with host buffers: K kc_forward calls
         (token and position in, the [vocab] float logits out to the host, the
         reference's ml_bench loop with its host argmax), wall clock
  tp     BASELINE config 4 (Llama-3-8B shape, Q8_0) decode at KV context
         --tp-ctx on this one GPU: the N = 1 point of the tensor-parallel curve
  extras decode at KV 128/1024/4096 and with F16/Q8 caches, configs 0 and 1
         (prompt + greedy decode as BASELINE runs them), config 3 (prefill at
         128/512/2048 tokens, then 64 decode steps), the CPU baseline

N > 1 (torchrun, one process per GPU): BASELINE config 4 decode at KV context
--tp-ctx, tensor parallel over the N GPUs (one model across them, the O and
down partial sums exchanged inside the step kernel over NVLink; sub-2B models
do not shard profitably and are reported at N = 1 only). value = tok/s of the
one token stream (max over ranks of the CUDA-event time), scaling "strong";
its N = 1 counterpart is the `tp` object of the N = 1 line.

--impl reference times the reference's own CPU build (oracle/_ref: the
reference's sources compiled unchanged; its best ISA for the host, all host
threads) on the same workload and config as the device arm at that N, rank 0
alone: the decode of K steps repeated --repeats times, the median reported.
That process loads no library of this repository: the model file is written
by the `mlbgen` command in a child process when missing, and its header is
read with struct.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "isa-lm_b200"))

P = argparse.ArgumentParser()
P.add_argument("--gpus", type=int, default=1)
P.add_argument("--steps", type=int, default=128)
P.add_argument("--warmup", type=int, default=8)
P.add_argument("--impl", choices=("ours", "reference"), default="ours")
P.add_argument("--config", default="cfg2")
P.add_argument("--ctx", type=int, default=1024)
P.add_argument("--no-extras", action="store_true", help="skip the sweeps, configs 0/1/3, TP1 and the CPU baseline")
P.add_argument("--tp-config", default="cfg4", help="model of the tensor-parallel decode ('none' to skip at N=1)")
P.add_argument("--tp-ctx", type=int, default=2048)
P.add_argument("--repeats", type=int, default=5, help="timed repeats of the CPU reference's decode")
ARGS = P.parse_args()

RANK = int(os.environ.get("RANK", "0"))
WORLD = int(os.environ.get("WORLD_SIZE", "1"))
LOCAL = int(os.environ.get("LOCAL_RANK", "0"))
# one GPU per rank: device LOCAL_RANK; every device stays visible, since a
# tensor-parallel rank maps the other ranks' exchange buffers (CUDA IPC)
_VIS = os.environ.get("CUDA_VISIBLE_DEVICES")
PHYS_DEV = (_VIS.split(",") if _VIS else [str(i) for i in range(64)])[LOCAL]

MODEL_DIR = os.environ.get("KRAFLA_MODEL_DIR", os.path.join(ROOT, "_models"))
PEAKS_PATH = os.path.join(ROOT, "MEASURED_PEAKS.json")
L2_NOTE = "weights larger than the 126 MB L2: streamed from HBM every step, no flush needed"


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def peaks():
    try:
        with open(PEAKS_PATH) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def bf16_peak():
    """Measured dense bf16 TFLOP/s (burst), else the pool's earlier figure."""
    try:
        with open(PEAKS_PATH) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    except (OSError, KeyError, ValueError):
        return 1590.0, "fallback"


def layer_macs(cfg):
    """Multiply-adds of one token through the layers' projections (prefill
    without the classifier): sum of rows * cols over wq wk wv wo w1 w2 w3."""
    d, h, qd, kvd = cfg["dim"], cfg["hidden_dim"], cfg["q_dim"], cfg["kv_dim"]
    return cfg["n_layers"] * (qd * d + 2 * kvd * d + d * qd + 3 * h * d)


def model_bytes_per_token(cfg, ctx, kv_bytes=4.0):
    """Algorithmic HBM bytes of one decode token: every quantized matrix (quants
    + f16 scales) once, the norm weights, the embedding row, and the KV rows
    attended (kv_bytes per element: 4 F32, 2 F16, 1 + 4/head_dim Q8 with its
    per-row scale)."""
    d, L, h, v = cfg["dim"], cfg["n_layers"], cfg["hidden_dim"], cfg["vocab"]
    qd, kvd = cfg["q_dim"], cfg["kv_dim"]
    wt, mask = cfg["wtype"], cfg["q8_mask"]

    def mat(rows, cols, bits):
        q8 = wt == 1 or (mask & bits)
        return rows * cols * (1 if q8 else 0.5) + rows * cols / 32 * (2 if cfg["scale_f16"] else 4)

    per_layer = (mat(qd, d, 4) + mat(kvd, d, 4) + mat(kvd, d, 8) + mat(d, qd, 16) + 2 * mat(h, d, 32) + mat(d, h, 64)
                 + 2 * d * 4)
    shared = cfg.get("shared", 0)
    cls = mat(v, d, 1 | 2 if shared else 2)
    emb = d * (1 if (wt == 1 or mask & 1) else 0.5)
    kv = 2 * L * ctx * kvd * kv_bytes
    return L * per_layer + cls + emb + kv


class Clocks:
    """nvidia-smi samples during the timed region (SM clock, throttle reasons)."""
    Q = ("clocks.sm,clocks.max.sm,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self):
        self.samples, self.stop = [], threading.Event()

    def __enter__(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", PHYS_DEV, f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "100"],
                                      stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.p = None
        return self

    def _read(self):
        for line in self.p.stdout:
            self.samples.append([s.strip() for s in line.split(",")])

    def __exit__(self, *a):
        if self.p:
            time.sleep(0.25)
            self.p.terminate()
            self.p.wait(timeout=5)

    def summary(self):
        sm = [float(s[0]) for s in self.samples if len(s) >= 7 and s[0].replace(".", "").isdigit()]
        mx = [float(s[1]) for s in self.samples if len(s) >= 7 and s[1].replace(".", "").isdigit()]
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({n for s in self.samples if len(s) >= 7 for n, v in zip(names, s[3:7]) if v == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(sm)}


def dist_init():
    if WORLD == 1:
        return None
    import datetime
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(LOCAL)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    return dist


def dist_max(dist, v):
    if dist is None:
        return v
    import torch
    t = torch.tensor([float(v)], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def prompt_tokens(vocab, n, seed=1234):
    import numpy as np
    return np.random.default_rng(seed).integers(0, vocab, n).astype(np.int32)


def arm_config(name, ctx, world):
    """The workload both arms measure at this N (the `config` of their JSON lines, identical in both)."""
    if world == 1:
        work = f"{name} batch-1 greedy decode at KV context {ctx}"
    else:
        work = f"{name} batch-1 greedy decode at KV context {ctx}, tensor parallel over {world} GPUs"
    return {"workload": work, "baseline_config": name, "ctx": ctx, "batch": 1, "kv_cache": "f32",
            "parallelism": f"tp{world}" if world > 1 else "single device", "inputs": L2_NOTE}


# ---------------------------------------------------------------- the CPU reference

def cpu_reference(path, vocab, ctx, steps, warmup, repeats, prompt_seed=1234):
    """The reference's best CPU build on this host (oracle/_ref), all host
    threads: prefill ctx - 1 prompt tokens, `warmup` greedy steps from the last
    prompt token, then `repeats` timed runs of `steps` greedy decode steps from
    the same token and position (app/ml_bench.c:120-131's loop), median."""
    import ctypes as C
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    ref = oracle.RefBuild()
    h = ref.open(path, os.cpu_count() or 1, 0, True)
    try:
        toks = prompt_tokens(vocab, ctx, prompt_seed)
        tp = ref.L.ref_time_prefill(h, toks.ctypes.data_as(C.c_void_p), ctx - 1, 0)
        out = (C.c_int * max(steps, warmup, 1))()
        tok, pos = int(toks[-1]), ctx - 1
        if warmup:
            if ref.L.ref_decode_greedy(h, tok, pos, warmup, out) < 0:
                raise RuntimeError("reference decode failed")
            tok, pos = int(out[warmup - 1]), pos + warmup
        rates = []
        for _ in range(max(1, repeats)):
            t = ref.L.ref_decode_greedy(h, tok, pos, steps, out)
            if t <= 0:
                raise RuntimeError("reference decode failed")
            rates.append(steps / t)
        threads = ref.L.ref_threads(h)
    finally:
        ref.L.ref_close(h)
    return {"decode_tok_s": statistics.median(rates), "decode_tok_s_min": min(rates),
            "decode_tok_s_max": max(rates), "repeats": len(rates), "prefill_tok_s": (ctx - 1) / tp,
            "cores": threads, "isa": ref.isa,
            "sample": f"{ctx - 1}-token prefill, {warmup} warm-up steps, then {len(rates)} x {steps} greedy decode "
                      f"steps from KV context {ctx - 1 + warmup} (median)"}


def reference_arm():
    """--impl reference: rank 0 alone, on the host cores, no process group, no GPU."""
    if RANK != 0:
        return
    import krafla_models as km
    K, W = ARGS.steps, ARGS.warmup
    name, want_ctx = (ARGS.config, ARGS.ctx) if WORLD == 1 else (ARGS.tp_config, ARGS.tp_ctx)
    path = km.ensure_model(name, MODEL_DIR)   # mlbgen, a child process, when the file is missing
    hdr = km.read_header(path)
    ctx = min(want_ctx, hdr["max_seq"] - K - W - 1)
    r = cpu_reference(path, hdr["vocab"], ctx, K, W, ARGS.repeats)
    v = round(r["decode_tok_s"], 3)
    line = {"metric": "batch-1 decode tok/s", "value": v, "unit": "tok/s", "impl": "reference", "n_gpus": WORLD,
            "steps": K, "warmup": W, "ms_per_step": round(1000.0 / r["decode_tok_s"], 3), "higher_is_better": True,
            "scaling": "strong" if WORLD > 1 else "weak", "vs_baseline": None, "dtype": "int8 dot, f32 accumulate",
            "data": "synthetic (seeded N(0,0.02) weights, uniform prompt ids)",
            "config": arm_config(name, ctx, WORLD),
            "cpu_baseline": {"value": v, "unit": "tok/s", "cores": r["cores"], "kind": "reference", "isa": r["isa"],
                             "sample": r["sample"], "min": round(r["decode_tok_s_min"], 3),
                             "max": round(r["decode_tok_s_max"], 3)},
            "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "prefill_tok_s": round(r["prefill_tok_s"], 1)}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- the device arm

def e2e_forward(kb, st, vocab, tok, pos, W, K, dist):
    """K kc_forward calls through the C ABI (the logits copied to the state's
    host buffer, the host argmax over it), after W untimed; wall clock, max over ranks."""
    import numpy as np
    fwd = kb.lib().kc_forward

    def step(t, p):
        ptr = fwd(st._h, t, p)
        if not ptr:
            raise RuntimeError("kc_forward failed: " + kb.what_detail())
        return int(np.argmax(np.ctypeslib.as_array(ptr, shape=(vocab,))))

    for _ in range(W):
        tok, pos = step(tok, pos), pos + 1
    if dist is not None:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(K):
        tok, pos = step(tok, pos), pos + 1
    return K / dist_max(dist, time.perf_counter() - t0)


def tp_state(kb, dist, name):
    """Model `name` sharded over the WORLD ranks (whole at WORLD 1) and a connected state."""
    if RANK == 0:
        path = kb.ensure_model(name, MODEL_DIR)
    if dist is not None:
        dist.barrier()
        path = kb.ensure_model(name, MODEL_DIR)
    t_load = time.perf_counter()
    model = kb.Model(path, upload=False)
    if WORLD > 1:
        model.shard(RANK, WORLD)
    st = kb.State(model)   # uploads this rank's share, then the state arena
    load_s = dist_max(dist, time.perf_counter() - t_load)
    if WORLD > 1:
        st.tp_connect(kb.exchange_handles(st.tp_handle(), dist))
    cfg = model.config
    cfg["shared"] = kb.CONFIGS[name].get("shared", 0)
    return model, st, cfg, load_s


def tp_release(dist, model, st):
    if dist is not None:
        dist.barrier()   # every rank's kernels are done before any exchange buffer goes
    st.free()
    model.free()
    if dist is not None:
        dist.barrier()


def tp_decode(kb, dist, K, W, hbm_peak, clocks=None):
    """--tp-config decode at KV context --tp-ctx over the WORLD ranks
    (kc_model_shard + kc_tp_connect); None when skipped."""
    name = ARGS.tp_config
    if name == "none" or name not in kb.CONFIGS:
        return None
    model, st, cfg, load_s = tp_state(kb, dist, name)
    ctx = min(ARGS.tp_ctx, cfg["max_seq"] - K - W - 1)
    toks = prompt_tokens(cfg["vocab"], ctx, seed=99)
    st.prefill(toks[:-1], 0)
    if dist is not None:
        dist.barrier()
    if clocks is not None:
        with clocks:
            ms = st.time_decode(int(toks[-1]), ctx - 1, W, K)
            if dist is not None:
                dist.barrier()
    else:
        ms = st.time_decode(int(toks[-1]), ctx - 1, W, K)
    ms = dist_max(dist, ms)
    tok_s = K / (ms / 1000.0)
    bpt = model_bytes_per_token(cfg, ctx - 1 + W + K // 2)
    e2e = None
    if WORLD > 1:   # the drop-in call on every rank, logits to the host
        st.prefill(toks[:-1], 0)
        e2e = e2e_forward(kb, st, cfg["vocab"], int(toks[-1]), ctx - 1, W, K, dist)
    tp_release(dist, model, st)
    return {"config": name, "workload": f"{name} batch-1 greedy decode at KV context {ctx}, tensor parallel",
            "ctx": ctx, "parallelism": f"tp{WORLD}", "n_gpus": WORLD, "scaling": "strong",
            "tok_s": round(tok_s, 2), "ms_per_token": round(ms / K, 4), "device_ms": ms, "steps": K, "warmup": W,
            "bytes_per_token": int(bpt), "load_s": round(load_s, 3),
            "hbm_frac_per_gpu": round(bpt / WORLD * tok_s / 1e9 / hbm_peak, 4), "e2e_tok_s": e2e,
            "exchange": "O and down partials as tagged 64-bit NVLink peer stores inside the step kernel "
                        "(no NCCL on the token path)"}


def tp_arm(kb, dist):
    """N > 1: the headline is the tensor-parallel decode of --tp-config."""
    hbm_peak, peak_kind = peaks()
    K, W = ARGS.steps, ARGS.warmup
    clk = Clocks()
    tp = tp_decode(kb, dist, K, W, hbm_peak, clocks=clk)
    if RANK == 0:
        per_gpu = tp["bytes_per_token"] / WORLD
        achieved = per_gpu * tp["tok_s"] / 1e9
        line = {"metric": "batch-1 decode tok/s", "value": tp["tok_s"], "unit": "tok/s", "n_gpus": WORLD,
                "steps": K, "warmup": W, "ms_per_step": tp["ms_per_token"], "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "int8 dot (dp4a), f32 accumulate",
                "data": "synthetic (seeded N(0,0.02) weights, uniform prompt ids)",
                "config": arm_config(tp["config"], tp["ctx"], WORLD),
                "roofline": {"bound": "hbm", "kernel": "step_kernel (tensor-parallel rank, one launch for K steps)",
                             "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                             "frac": round(achieved / hbm_peak, 4), "peak_kind": peak_kind, "traffic": None,
                             "per": "GPU (each rank streams 1/N of the weights and KV)"},
                "e2e": {"value": round(tp["e2e_tok_s"], 2), "unit": "tok/s", "h2d_bytes_per_step": 32,
                        "d2h_bytes_per_step": 4 * 128256 + 32,
                        "path": "kc_forward per token on every rank (logits to host) + host argmax"},
                "gpu_launches": 1, "steps_per_launch": K, "clocks": clk.summary(), "tp": tp}
        print(json.dumps(line), flush=True)


def decode_line(kb, name, prompt_len, n_decode, hbm_peak):
    """BASELINE's run of config `name` (configs 0 and 1): a prompt of uniform ids,
    then greedy decode on the device, one launch timed by CUDA events; plus the
    reference's CPU build on the same model and sample."""
    path = kb.ensure_model(name, MODEL_DIR)
    model = kb.Model(path)
    cfg = model.config
    cfg["shared"] = kb.CONFIGS[name].get("shared", 0)
    st = kb.State(model)
    toks = prompt_tokens(cfg["vocab"], prompt_len, seed=5)
    st.prefill(toks[:-1], 0)
    ms = st.time_decode(int(toks[-1]), prompt_len - 1, 3, n_decode)
    st.prefill(toks[:-1], 0)
    e2e = e2e_forward(kb, st, cfg["vocab"], int(toks[-1]), prompt_len - 1, 3, n_decode, None)
    st.free()
    model.free()
    tok_s = n_decode / (ms / 1000.0)
    bpt = model_bytes_per_token(cfg, prompt_len + n_decode // 2)
    out = {"workload": f"{name}: {prompt_len}-token prompt, then {n_decode} greedy decode steps",
           "tok_s": round(tok_s, 1), "e2e_tok_s": round(e2e, 1), "bytes_per_token": int(bpt),
           "hbm_frac": round(bpt * tok_s / 1e9 / hbm_peak, 4)}
    if name == "cfg0":
        out["note"] = "16 MB of weights stay in L2: launch- and latency-bound, HBM fraction not meaningful"
    try:
        r = cpu_reference(path, cfg["vocab"], prompt_len, n_decode, 3, 3, prompt_seed=5)
        out["cpu_reference"] = {"tok_s": round(r["decode_tok_s"], 1), "cores": r["cores"], "isa": r["isa"],
                                "sample": r["sample"]}
    except Exception as e:   # the reference build needs a compatible host CPU
        out["cpu_reference"] = {"error": str(e)}
    return out


def main():
    if ARGS.impl == "reference":
        reference_arm()
        return
    import numpy as np
    import krafla_b200 as kb
    dist = dist_init()
    kb.set_device(LOCAL)
    if WORLD > 1:
        tp_arm(kb, dist)
        dist.barrier()
        dist.destroy_process_group()
        return

    hbm_peak, peak_kind = peaks()
    path = kb.ensure_model(ARGS.config, MODEL_DIR)
    K, W = ARGS.steps, ARGS.warmup
    t_load = time.perf_counter()
    model = kb.Model(path)   # map + validate the .mlb, upload (file -> pinned -> HBM)
    load_s = time.perf_counter() - t_load
    load_bytes = int(model.device_bytes)
    cfg = model.config
    cfg["shared"] = kb.CONFIGS[ARGS.config].get("shared", 0)
    ctx = min(ARGS.ctx, cfg["max_seq"] - K - W - 1)
    st = kb.State(model)
    toks = prompt_tokens(cfg["vocab"], ctx)
    st.prefill(toks[:-1], 0)
    start_tok, start_pos = int(toks[-1]), ctx - 1

    # --- value: device time of K steps in one launch (CUDA events on the launching stream)
    with Clocks() as clk:
        ms = st.time_decode(start_tok, start_pos, W, K)
    value = K / (ms / 1000.0)
    bpt = model_bytes_per_token(cfg, ctx - 1 + W + K // 2)

    # --- e2e: the drop-in C ABI with host buffers, ml_bench's loop (app/ml_bench.c:125-131)
    st.prefill(toks[:-1], 0)
    e2e = e2e_forward(kb, st, cfg["vocab"], start_tok, start_pos, W, K, None)
    # device-resident greedy loop through the C ABI (host tokens in and out)
    st.prefill(toks[:-1], 0)
    t0 = time.perf_counter()
    st.generate_greedy(start_tok, start_pos, K)
    greedy_s = time.perf_counter() - t0

    # --- roofline of the dominant kernel: the step kernel is the only kernel of the timed
    # region (one cooperative launch runs the K steps), so its achieved bandwidth is the
    # algorithmic bytes of K steps over the same CUDA-event time
    achieved = bpt * K / (ms / 1000.0) / 1e9
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tpath):
        with open(tpath) as f:
            t = json.load(f).get(f"{ARGS.config}:step_kernel")
        if t:   # DRAM bytes of one captured step, times the K steps of the timed launch
            traffic = int(t["bytes_per_step"]) * K
    st.prefill(toks[:-1], 0)
    tl = st.step_timeline(start_tok, start_pos)
    d = np.diff(tl) / 1000.0
    L = cfg["n_layers"]
    phases = {}
    if len(d) >= 5 * L + 1:
        per = d[:5 * L].reshape(L, 5)
        phases = {n: round(float(v), 2) for n, v in zip(("qkv", "attention", "wo", "ffn_up", "ffn_down"), per.sum(0))}
        phases["classifier"] = round(float(d[5 * L:].sum()), 2)

    extras = {}
    if not ARGS.no_extras:
        sweep = {}
        for c in (128, 1024, 4096):
            c2 = min(c, cfg["max_seq"] - 34)
            st.prefill(prompt_tokens(cfg["vocab"], c2)[:-1], 0)
            m2 = st.time_decode(1, c2 - 1, 2, 32)
            b2 = model_bytes_per_token(cfg, c2 + 18)
            sweep[str(c)] = {"tok_s": round(32 / (m2 / 1000), 1),
                             "hbm_frac": round(b2 * 32 / (m2 / 1000) / 1e9 / hbm_peak, 4)}
        extras["decode_by_context"] = sweep
        # the same decode with the F16 and Q8 caches (row f1): fewer KV bytes per token
        kvs = {}
        for kvname, kvt, kvb in (("f16", kb.F16, 2.0), ("q8", kb.Q8_0, 1.0 + 4.0 / cfg["head_dim"])):
            try:
                sk = kb.State(model, kv_type=kvt)
                row = {}
                for c in (1024, 4096):
                    c2 = min(c, cfg["max_seq"] - 34)
                    sk.prefill(prompt_tokens(cfg["vocab"], c2)[:-1], 0)
                    m2 = sk.time_decode(1, c2 - 1, 2, 32)
                    b2 = model_bytes_per_token(cfg, c2 + 18, kvb)
                    row[str(c)] = {"tok_s": round(32 / (m2 / 1000), 1),
                                   "hbm_frac": round(b2 * 32 / (m2 / 1000) / 1e9 / hbm_peak, 4)}
                sk.free()
                kvs[kvname] = row
            except Exception as e:   # a KV type this model's head layout cannot use
                kvs[kvname] = {"error": str(e)}
        extras["decode_by_kv_cache"] = kvs
        # sampled generation on the device (top-k 40, top-p 0.95, T 0.8, penalty 1.1 over 64): step + sample kernel
        # per token, no logits copy
        smp = kb.Sampler(st, temperature=0.8, topk=40, topp=0.95, repeat_penalty=1.1, repeat_last_n=64, seed=1)
        st.prefill(toks[:-1], 0)
        t0 = time.perf_counter()
        st.generate_sampled(smp, start_tok, start_pos, 32)
        extras["e2e_sampled_device"] = {"value": round(32 / (time.perf_counter() - t0), 2), "unit": "tok/s",
                                        "sampler": "T 0.8, top-k 40, top-p 0.95, repeat penalty 1.1 / 64"}
        smp.free()

        # config 3: prefill through the batched tensor-core path, wall clock around the
        # whole host call (best of 3, after one call that packs the weights), then 64
        # decode steps after the 2048-token prompt
        pre, pre_roof = {}, {}
        st.prefill(prompt_tokens(cfg["vocab"], 128, seed=7), 0)
        ops_tok = 2.0 * layer_macs(cfg)
        bf16, bf16_kind = bf16_peak()
        int8_peak = 2.0 * bf16
        for n in (128, 512, 2048):
            pt = prompt_tokens(cfg["vocab"], n, seed=7)
            best = None
            for _ in range(3):
                t0 = time.perf_counter()
                st.prefill(pt, 0)
                dt = time.perf_counter() - t0
                best = dt if best is None else min(best, dt)
            pre[str(n)] = round(n / best, 1)
            pre_roof[str(n)] = round(ops_tok * n / best / 1e12 / int8_peak, 4)
        extras["prefill_tok_s"] = pre
        extras["prefill_roofline"] = {"bound": "tensor", "unit": "TOP/s", "peak": int8_peak,
                                      "peak_kind": f"2x {bf16_kind} bf16 dense (the int8 rate of B200)",
                                      "ops_per_token": ops_tok, "frac_by_prompt": pre_roof}
        pt = prompt_tokens(cfg["vocab"], 2048, seed=7)
        st.prefill(pt[:-1], 0)
        m3 = st.time_decode(int(pt[-1]), 2047, 0, 64)
        b3 = model_bytes_per_token(cfg, 2048 + 32)
        extras["cfg3_decode_after_prefill"] = {"workload": "cfg3: 2048-token prefill, then 64 greedy decode steps",
                                               "tok_s": round(64 / (m3 / 1000), 1),
                                               "hbm_frac": round(b3 * 64 / (m3 / 1000) / 1e9 / hbm_peak, 4)}
    st.free()
    model.free()
    if not ARGS.no_extras:
        extras["cfg0"] = decode_line(kb, "cfg0", 16, 128, hbm_peak)
        extras["cfg1"] = decode_line(kb, "cfg1", 32, 256, hbm_peak)
        try:   # the same sample as --impl reference
            extras["cpu_baseline"] = cpu_reference(path, cfg["vocab"], ctx, K, W, ARGS.repeats)
        except Exception as e:   # the reference build needs a compatible host CPU
            extras["cpu_baseline"] = {"error": str(e)}
    tp = None if ARGS.no_extras else tp_decode(kb, None, min(K, 64), max(W, 3), hbm_peak)

    cpu = extras.get("cpu_baseline", {})
    line = {
        "metric": "batch-1 decode tok/s", "value": round(value, 2), "unit": "tok/s", "n_gpus": 1,
        "steps": K, "warmup": W, "ms_per_step": round(ms / K, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8 dot (dp4a), f32 accumulate",
        "data": "synthetic (seeded N(0,0.02) weights, uniform prompt ids)",
        "config": arm_config(ARGS.config, ctx, 1),
        "hbm_roofline_frac": round(bpt * value / 1e9 / hbm_peak, 4),
        "bytes_per_token": int(bpt),
        "roofline": {"bound": "hbm", "kernel": "step_kernel (whole decode step, one launch for K steps)",
                     "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                     "frac": round(achieved / hbm_peak, 4), "peak_kind": peak_kind, "traffic": traffic},
        "e2e": {"value": round(e2e, 2), "unit": "tok/s", "h2d_bytes_per_step": 32,
                "d2h_bytes_per_step": 4 * cfg["vocab"] + 32,
                "path": "kc_forward per token (logits to host) + host argmax"},
        "e2e_greedy_device": {"value": round(K / greedy_s, 2), "unit": "tok/s",
                              "h2d_bytes_per_step": round(32 / K, 2), "d2h_bytes_per_step": 4},
        "gpu_launches": 1,
        "steps_per_launch": K,
        "clocks": clk.summary(),
        "step_phase_us": phases,
    }
    if cpu and "decode_tok_s" in cpu:
        line["cpu_baseline"] = {"value": round(cpu["decode_tok_s"], 3), "unit": "tok/s", "cores": cpu["cores"],
                                "kind": "reference", "isa": cpu["isa"], "sample": cpu["sample"],
                                "min": round(cpu["decode_tok_s_min"], 3), "max": round(cpu["decode_tok_s_max"], 3),
                                "prefill_tok_s": round(cpu["prefill_tok_s"], 1)}
    elif cpu:
        line["cpu_baseline"] = cpu
    line["model_load"] = {"config": ARGS.config, "seconds": round(load_s, 3), "device_bytes": load_bytes,
                          "path": "kc_model_load + kc_model_upload"}
    for k in ("decode_by_context", "decode_by_kv_cache", "e2e_sampled_device", "prefill_tok_s", "prefill_roofline",
              "cfg3_decode_after_prefill", "cfg0", "cfg1"):
        if k in extras:
            line[k] = extras[k]
    if tp is not None:
        line["tp"] = tp
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
