"""Benchmark of the PGF training step (fwd + bwd + AdamW) on B200.

Workload (default): the 8-layer PGF Mamba language model of the reference's training scripts at
d_model 256 / d_state 16 / d_ff 1024 / vocab 50257 (reference SSM variant, untied embedding and
LM head as in train_wikitext_rebuttal.py:58-77), ONE sequence of L = 1,048,576 tokens with PGF
block size 4096, synthetic Zipf(1.1) token ids, bf16 activations, fp32 weights and AdamW.  On N GPUs
(one process each) the default shards that one sequence across the GPUs (contiguous segments,
boundary-state hand-off between segments, one gradient all-reduce): the total work is fixed (strong
scaling).  --parallel dp runs one such sequence per GPU instead (weak scaling).

The same line carries, under "mamba_standard", the same measurement of the Mamba-standard model of
the benchmark configurations (d_inner 512, d_conv 4, dt_rank 16, per-channel A, final RMSNorm, tied
head) on the same sequence and GPUs, which the reference has no code for (--no-std-companion skips
it; --variant std makes it the headline).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--seq-len L] [--impl b200|reference]

--impl reference times the reference's PGF step restated on the CPU (the oracle, float32, all host
threads) on a bounded prefix of the same sequence (--cpu-sample-len tokens, same model and block
size), K steps after W warm-ups.  Prints one JSON line on rank 0.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import torch  # noqa: E402

def metric_of(a) -> str:
    return f"fwd+bwd tokens/s ({a.layers}-layer PGF Mamba LM)"
UNIT = "tokens/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--seq-len", type=int, default=1048576,
                    help="tokens of one sequence (sp: the one sequence sharded over the GPUs; dp: one per GPU)")
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--layers", type=int, default=8)
    ap.add_argument("--d-model", type=int, default=256)
    ap.add_argument("--d-ff", type=int, default=1024)
    ap.add_argument("--dt-rank", type=int, default=16, help="Mamba-standard variant: dt_proj rank")
    ap.add_argument("--vocab", type=int, default=50257)
    ap.add_argument("--block-size", type=int, default=4096)
    ap.add_argument("--dtype", default="bf16", choices=["bf16", "fp32"])
    ap.add_argument("--cpu-sample-len", type=int, default=2048,
                    help="tokens of the sequence prefix one CPU step processes (reference arm, cpu_baseline)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--variant", default="reference", choices=["reference", "std"],
                    help="reference: the reference's SSM block (d_inner = d_model); std: the Mamba-standard "
                         "block of the benchmark configurations (expand 2, d_conv 4, dt_rank 16, final "
                         "RMSNorm, tied LM head)")
    ap.add_argument("--component", default=None, choices=["rmsnorm", "ffn", "lmhead", "jvp", "scan", "all"],
                    help="component microbenchmarks instead of the LM step (RMSNorm [8,4096,1024]; FFN "
                         "1024-4096-1024 on 32768 tokens; LM head + CE d=1024, vocab 50257, 32768 tokens; "
                         "scan: one reference-variant SSM layer's saved forward and backward on one segment)")
    ap.add_argument("--stash", default="device", choices=["device", "host", "scan"],
                    help="where layer inputs wait for the backward: device memory, pinned host memory, or "
                         "device memory together with each layer's scan states (no scan recompute)")
    ap.add_argument("--no-std-companion", action="store_true",
                    help="skip the Mamba-standard model measured after the reference variant (key mamba_standard)")
    ap.add_argument("--no-graph", action="store_true",
                    help="time eager launches instead of the CUDA-graph captured step (1 GPU)")
    ap.add_argument("--parallel", default="sp", choices=["sp", "dp"],
                    help="N>1: sp = the one sequence of seq-len tokens sharded across the GPUs (state "
                         "hand-off between segments; strong scaling), dp = one sequence per GPU (weak)")
    return ap.parse_args()


def per_rank_len(a, world):
    """Tokens of the sequence each rank holds: its segment (sp) or its own sequence (dp)."""
    if world > 1 and a.parallel == "sp":
        if a.seq_len % world:
            raise SystemExit(f"--seq-len {a.seq_len} must split evenly over {world} GPUs")
        return a.seq_len // world
    return a.seq_len


def scaling_of(a, world):
    return "strong" if a.parallel == "sp" else "weak"


def config_of(a, world):
    var = ("reference SSM variant" if a.variant == "reference" else
           f"Mamba-standard variant (d_inner {2 * a.d_model}, d_conv 4, dt_rank {a.dt_rank}, final RMSNorm, "
           f"tied head)")
    seqs = a.batch * (world if a.parallel == "dp" else 1)
    where = (f"one sequence per GPU" if a.parallel == "dp" else
             (f"sharded over {world} GPUs ({a.seq_len // world} tokens each)" if world > 1 else "on one GPU"))
    return {
        "workload": f"{a.layers}-layer PGF Mamba LM ({var}), d_model {a.d_model}, d_state 16, d_ff {a.d_ff}, "
                    f"vocab {a.vocab}, B={a.batch} x L={a.seq_len} tokens {where}, PGF block {a.block_size}, "
                    f"{a.dtype} activations / fp32 weights + AdamW",
        "layers": a.layers, "d_model": a.d_model, "d_state": 16, "d_ff": a.d_ff, "vocab": a.vocab,
        "global_batch": seqs, "seq_len": a.seq_len, "pgf_block_size": a.block_size,
        "parallelism": f"{a.parallel}{world}",
        "ssm_variant": ("reference (d_inner = d_model, shared A)" if a.variant == "reference" else
                        "mamba-standard (d_inner 2 d_model, conv1d, gate, per-channel A)"),
        "l2": "per-step working set (weights, optimizer state, activations) > 126 MB L2; no explicit flush",
        "stash": a.stash,
        "optimizer": "AdamW (flat parameter buffer, libpgf kernels)",
    }


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        load = [s for s in sm if mx and s > 0.5 * mx] or sm
        return {"sm_mhz": statistics.median(load) if load else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------------------- CPU baseline
class CpuStep:
    """The oracle (CPU restatement of the reference's PGF LM step, float32, all host threads) on a
    bounded prefix of the benchmark sequence: the same model, vocabulary and PGF block size, the
    first cpu_sample_len tokens."""

    def __init__(self, a):
        from oracle import pgf_oracle as O
        self.O = O
        self.threads = os.cpu_count() or 1
        torch.set_num_threads(self.threads)
        g = torch.Generator().manual_seed(0)
        self.blocks = [O.block_init(a.d_model, 16, a.d_ff, g) for _ in range(a.layers)]
        self.emb = torch.randn(a.vocab, a.d_model, generator=g) * 0.02
        self.lmw = torch.randn(a.vocab, a.d_model, generator=g) * 0.02
        self.L = a.cpu_sample_len
        ids = zipf_ids(self.L + 1, a.vocab, seed=100).reshape(1, self.L + 1)
        self.x, self.y = ids[:, :-1], ids[:, 1:]
        self.bs = a.block_size

    def __call__(self):
        self.O.lm_pgf_step(self.emb, self.lmw, self.blocks, self.x, self.y, self.bs)

    def sample(self, steps, warmup):
        return (f"the oracle's PGF step (fp32, no optimizer) of the same {len(self.blocks)}-layer model on the first "
                f"{self.L} tokens of the sequence (PGF block {self.bs}), {steps} timed steps after {warmup} warm-up, "
                f"{self.threads} host threads")


def cpu_baseline(a, kind="port", steps=3, warmup=1):
    """Bounded CPU sample (about 10-30 s of host work) reported beside the GPU arm."""
    st = CpuStep(a)
    for _ in range(warmup):
        st()
    t0 = time.perf_counter()
    for _ in range(steps):
        st()
    dt = time.perf_counter() - t0
    return {"value": st.L * steps / dt, "unit": UNIT, "cores": torch.get_num_threads(), "kind": kind,
            "sample": st.sample(steps, warmup)}


def run_reference(a, rank, world):
    """The reference arm: K timed CPU steps (after W warm-ups) of the bounded sample, rank 0 only."""
    if rank != 0:
        return
    st = CpuStep(a)
    for _ in range(a.warmup):
        st()
    t0 = time.perf_counter()
    for _ in range(a.steps):
        st()
    dt = time.perf_counter() - t0
    value = st.L * a.steps / dt
    cb = {"value": value, "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
          "sample": st.sample(a.steps, a.warmup)}
    line = {"metric": metric_of(a), "value": value, "unit": UNIT, "n_gpus": world, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": 1000.0 * dt / max(a.steps, 1),
            "higher_is_better": True, "scaling": scaling_of(a, world), "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (Zipf 1.1 token ids, random init)", "impl": "reference", "config": config_of(a, world),
            "cpu_baseline": cb,
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- GPU arm
# DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum) of the dominant kernels, from
# ncu captures on the 65536-token segment every launch of the default workload covers (8-layer
# reference variant, d 256, d_ff 1024, vocab 50257, bf16): the scan kernels one launch each from
# `bench.py --component scan`; gemm_tc and ce the mean over one step's launches of the group, the
# RMSNorm kernels the mean of two launches (the forward: one with and one without the residual),
# the others one launch each, from the 65536-token step.  Reported as `traffic` only for that workload.
TRAFFIC_DEFAULT = {"gemm_tc": 194297962, "ssm_main_bwd": 496966144, "ce": 1316357018, "ssm_chunk_fwd": 288500000,
                   "ssm_out_fwd": 230101748, "ssm_chunk_bwd": 114800000, "ssm_compose": 8940480,
                   "rmsnorm_fwd": 60879232, "rmsnorm_bwd": 115444608, "adamw": 395415392}
# Warp instructions per launch of the scan backward on that segment (smsp__inst_executed.sum, same
# capture): the kernel is bound by instruction issue, so its compute roofline is issue rate.
MAIN_BWD_WARP_INSTS = 517951488
SMS, ISSUE_PER_SM_CLK = 148, 4


def default_workload(a, world):
    """The default LM workload, whose per-launch shapes the captures above measured (sequences of
    65536 tokens or longer run in 65536-token segments)."""
    per_rank = a.seq_len // world if (world > 1 and a.parallel == "sp") else a.seq_len
    return (a.variant == "reference" and a.layers == 8 and a.d_model == 256 and a.d_ff == 1024 and a.vocab == 50257
            and a.batch == 1 and per_rank % 65536 == 0 and a.dtype == "bf16" and a.block_size == 4096)


def issue_roofline(ms_per_launch, sm_mhz):
    """The scan backward against the SMs' instruction-issue peak (4 warp instructions per SM per clock)."""
    ach = MAIN_BWD_WARP_INSTS / (ms_per_launch / 1e3) / 1e9
    peak = SMS * ISSUE_PER_SM_CLK * sm_mhz / 1e3
    return {"bound": "issue", "achieved": ach, "peak": peak, "unit": "G warp-instructions/s", "frac": ach / peak,
            "kernel": "ssm_main_bwd", "warp_instructions_per_launch": MAIN_BWD_WARP_INSTS,
            "peak_source": f"{SMS} SMs x {ISSUE_PER_SM_CLK} per clock at the sampled {sm_mhz:.0f} MHz"}


def roofline_entry(name, ms_total, n, work_total, traffic=None):
    """Achieved rate of one kernel (algorithmic work / its average launch time measured with CUDA
    events in the timed region) against MEASURED_PEAKS.json (sustained bf16 figure: the kernels run
    inside a long step)."""
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        pass
    src = "measured" if peaks else "fallback"
    t = ms_total / n / 1e3
    if name.startswith("gemm") or name == "ce":
        peak = peaks.get("bf16_tflops_sustained", 1400.0)
        ach = work_total / n / t / 1e12
        return {"bound": "tensor", "achieved": ach, "peak": peak, "unit": "TFLOP/s", "frac": ach / peak,
                "traffic": traffic, "kernel": name, "peak_source": src + " (bf16 sustained)",
                "work_per_launch": work_total / n, "ms_per_launch": t * 1e3}
    peak = peaks.get("hbm_gbs", 6650.0)
    ach = work_total / n / t / 1e9
    return {"bound": "hbm", "achieved": ach, "peak": peak, "unit": "GB/s", "frac": ach / peak,
            "traffic": traffic, "kernel": name, "peak_source": src,
            "work_per_launch": work_total / n, "ms_per_launch": t * 1e3}


def main():
    a = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if a.impl == "reference":
        run_reference(a, rank, world)
        return
    if a.component:
        run_components(a)
        return
    run_gpu(a, rank, world, local_rank)


def _time(fn, steps, warmup):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def run_components(a):
    """Component microbenchmarks: one JSON line each (rates against MEASURED_PEAKS.json)."""
    from icml_b200 import ops
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        pass
    hbm, tf = peaks.get("hbm_gbs", 6650.0), peaks.get("bf16_tflops", 1590.0)
    dev = torch.device("cuda")
    g = torch.Generator(device="cpu").manual_seed(0)
    which = ["rmsnorm", "ffn", "lmhead", "jvp", "scan"] if a.component == "all" else [a.component]
    if "jvp" in which:
        run_jvp_components(a, hbm, tf, g, dev)
        which = [w for w in which if w != "jvp"]
    if "scan" in which:
        run_scan_component(a, g, dev)
        which = [w for w in which if w != "scan"]
    for dt_name, dt in (("bf16", torch.bfloat16), ("fp32", torch.float32)):
        if "rmsnorm" in which:
            x = torch.randn(8, 4096, 1024, generator=g).to(dev, dt)
            gy = torch.randn(8, 4096, 1024, generator=g).to(dev, dt)
            w = (1 + 0.02 * torch.randn(1024, generator=g)).to(dev)
            ms = _time(lambda: (ops.rmsnorm_fwd(x, w, 1e-5), ops.rmsnorm_bwd(x, gy, w, 1e-5)), a.steps, a.warmup)
            by = 8 * 4096 * 1024 * x.element_size() * 5  # read x twice, g; write y, dx
            print(json.dumps({"metric": "RMSNorm fwd+bwd [8,4096,1024] eps 1e-5", "value": by / ms / 1e6,
                              "unit": "GB/s", "dtype": dt_name, "ms": ms,
                              "roofline": {"bound": "hbm", "achieved": by / ms / 1e6, "peak": hbm,
                                           "frac": by / ms / 1e6 / hbm}}), flush=True)
        # the wide FFN of the component configuration, and the LM's own FFN on one 65536-token segment
        for T, d, dh in ((32768, 1024, 4096), (65536, 256, 1024)):
            if "ffn" not in which or (dt_name == "fp32" and d == 256):
                continue
            x = torch.randn(T, d, generator=g).to(dev, dt)
            gy = torch.randn(T, d, generator=g).to(dev, dt)
            W1 = (0.02 * torch.randn(dh, d, generator=g)).to(dev)
            W2 = (0.02 * torch.randn(d, dh, generator=g)).to(dev)
            b1, b2 = torch.zeros(dh, device=dev), torch.zeros(d, device=dev)
            ms = _time(lambda: (ops.ffn_fwd(x, W1, b1, W2, b2), ops.ffn_bwd(x, gy, W1, b1, W2)), a.steps, a.warmup)
            fl = 8 * 2.0 * T * d * dh  # fwd 2 + backward 6 (incl. the recomputed forward)
            print(json.dumps({"metric": f"FFN {d}-{dh}-{d} fwd+bwd, {T} tokens", "value": fl / ms / 1e9,
                              "unit": "TFLOP/s", "dtype": dt_name, "ms": ms,
                              "roofline": {"bound": "tensor", "achieved": fl / ms / 1e9, "peak": tf,
                                           "frac": fl / ms / 1e9 / tf}}), flush=True)
        if "lmhead" in which:
            T, d, V = 32768, 1024, 50257
            h = torch.randn(T, d, generator=g).to(dev, dt)
            W = (0.02 * torch.randn(V, d, generator=g)).to(dev)
            tg = torch.randint(0, V, (T,), generator=g).to(dev)

            def step():
                _, lse = ops.lm_head_ce_fwd(h, W, tg)
                ops.lm_head_ce_bwd(h, W, tg, lse, 1.0 / T)
            ms = _time(step, max(1, a.steps // 3), max(1, a.warmup // 2))
            fl = 4 * 2.0 * T * V * d  # forward, recomputed logits, dW, dh
            print(json.dumps({"metric": "LM head + CE fwd+bwd, d 1024, vocab 50257, 32768 tokens",
                              "value": fl / ms / 1e9, "unit": "TFLOP/s", "dtype": dt_name, "ms": ms,
                              "roofline": {"bound": "tensor", "achieved": fl / ms / 1e9, "peak": tf,
                                           "frac": fl / ms / 1e9 / tf}}), flush=True)


def run_scan_component(a, g, dev):
    """The selective-scan layer of the reference variant (d_model x 16 states) on one 65536-token
    segment in bf16: the backward's saved forward (re-run, checkpoints) and the scan backward, the
    kernels the LM step launches per layer and segment.  One JSON line with each kernel's time per
    launch (libpgf's CUDA events) and its roofline against MEASURED_PEAKS.json."""
    import ctypes
    from icml_b200 import _lib, ops
    from icml_b200.train_singlemamba_optimized import SingleLayerMambaPGF, _cat_weights
    L = min(a.seq_len, 65536)
    torch.manual_seed(0)
    layer = SingleLayerMambaPGF(a.d_model, 16).to(dev)
    u = torch.randn(1, L, a.d_model, generator=g).to(dev, torch.bfloat16)
    gy = torch.randn(1, L, a.d_model, generator=g).to(dev, torch.bfloat16)
    W, b = _cat_weights(layer)

    def step():
        y, saved = ops.ssm_fwd_save(u, W, b, layer.A_log, layer.D, layer.scale)
        ops.ssm_bwd(u, gy, W, b, layer.A_log, layer.D, layer.scale, saved=saved)

    for _ in range(max(a.warmup, 1)):
        step()
    torch.cuda.synchronize()
    Lb = _lib.lib()
    Lb.pgf_profile(1)
    for _ in range(a.steps):
        step()
    torch.cuda.synchronize()
    Lb.pgf_profile(0)
    kernels = {}
    for i, nm in PROF_NAMES.items():
        c, t, w = ctypes.c_longlong(0), ctypes.c_double(0.0), ctypes.c_double(0.0)
        Lb.pgf_profile_read(i, ctypes.byref(c), ctypes.byref(t), ctypes.byref(w))
        if c.value:
            kernels[nm] = roofline_entry(nm, t.value, c.value, w.value)
    print(json.dumps({"metric": f"scan layer saved forward + backward, B=1 x L={L}, d {a.d_model}, 16 states, bf16",
                      "unit": "ms per launch", "steps": a.steps, "kernels": kernels}), flush=True)


def run_jvp_components(a, hbm, tf, g, dev):
    """Forward-mode operators: the Frechet operator's JVP at the reference scaling benchmark's model
    (d_model 256, d_state 16; bench_scaling.py:29-32), the FFN JVP and the RMSNorm JVP."""
    from icml_b200 import ops
    from icml_b200.pgf_mamba import FrechetMambaOperator
    L, D = a.seq_len, 256
    torch.manual_seed(0)
    m = FrechetMambaOperator(d_model=D, d_state=16).to(dev)
    u = (0.1 * torch.randn(L, D, generator=g)).to(dev)
    du = torch.randn(L, D, generator=g)
    du = (du / du.norm()).to(dev)
    ms = _time(lambda: m.pgf_forward(u, du), a.steps, a.warmup)
    by = L * D * 4 * 4  # read u, u_dot; write y, y_dot (float32)
    line = {"metric": "Frechet operator JVP tokens/s (d_model 256, d_state 16, y and y_dot)", "value": L / ms * 1e3,
            "unit": "tokens/s", "dtype": "fp32", "ms": ms, "config": {"workload": f"L={L} x d_model {D}"},
            "roofline": {"bound": "hbm", "achieved": by / ms / 1e6, "peak": hbm, "frac": by / ms / 1e6 / hbm,
                         "note": "the (state, tangent) scan is instruction-bound; bytes are its inputs/outputs"}}
    if not a.no_cpu_baseline:
        import time
        from oracle import jvp_oracle as J
        from tests.test_oracle_golden import frechet_params
        torch.set_num_threads(os.cpu_count() or 1)
        n = 512
        p = {k: v.detach().cpu().double() for k, v in
             frechet_params({k: v.detach().cpu() for k, v in m.state_dict().items()}).items()}
        uc, duc = u[:n].cpu().double(), du[:n].cpu().double()
        t0 = time.perf_counter()
        J.frechet_jvp(p, uc, duc)
        dt_ = time.perf_counter() - t0
        line["cpu_baseline"] = {"value": n / dt_, "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": "port",
                                "sample": f"the oracle's token-by-token JVP (float64) over the first {n} tokens"}
    print(json.dumps(line), flush=True)
    # state HVP trajectory of the reference SSM layer (train_singlemamba_optimized.py:563-685)
    from icml_b200.train_singlemamba_optimized import SingleLayerMambaPGF
    lay = SingleLayerMambaPGF(D, 16).to(dev)
    uh = torch.randn(1, L, D, generator=g).to(dev)
    th = torch.randn(1, L, D, generator=g).to(dev)
    vh = torch.randn(1, D, 16, generator=g).to(dev)
    ms = _time(lambda: lay.compute_state_hvp(uh, th, vh, 4096), a.steps, a.warmup)
    by = L * D * 16 * 4 + 2 * L * D * 4  # the (L, B, D, N) trajectory written, u and target read
    print(json.dumps({"metric": "SSM state-HVP trajectory tokens/s (d_model 256, d_state 16)", "value": L / ms * 1e3,
                      "unit": "tokens/s", "dtype": "fp32", "ms": ms, "config": {"workload": f"B=1 x L={L} x d {D}"},
                      "roofline": {"bound": "hbm", "achieved": by / ms / 1e6, "peak": hbm,
                                   "frac": by / ms / 1e6 / hbm}}), flush=True)
    T, d, dh = 32768, 1024, 4096
    for dt_name, dt in (("bf16", torch.bfloat16), ("fp32", torch.float32)):
        x = torch.randn(T, d, generator=g).to(dev, dt)
        xd = torch.randn(T, d, generator=g).to(dev, dt)
        ws = [(0.02 * torch.randn(*s_, generator=g)).to(dev) for s_ in ((dh, d), (dh, d), (dh,), (dh,), (d, dh),
                                                                       (d, dh), (d,), (d,))]
        ms = _time(lambda: ops.ffn_jvp(x, xd, *ws), a.steps, a.warmup)
        fl = 6 * 2.0 * T * d * dh  # z (1), z_dot over 2d (2), y (1), y_dot over 2 dh (2)
        print(json.dumps({"metric": "FFN JVP 1024-4096-1024, 32768 tokens", "value": fl / ms / 1e9, "unit": "TFLOP/s",
                          "dtype": dt_name, "ms": ms,
                          "roofline": {"bound": "tensor", "achieved": fl / ms / 1e9, "peak": tf,
                                       "frac": fl / ms / 1e9 / tf}}), flush=True)
        x3 = torch.randn(8, 4096, 1024, generator=g).to(dev, dt)
        xd3 = torch.randn(8, 4096, 1024, generator=g).to(dev, dt)
        w, wd = (1 + 0.02 * torch.randn(1024, generator=g)).to(dev), (0.02 * torch.randn(1024, generator=g)).to(dev)
        ms = _time(lambda: ops.rmsnorm_jvp(x3, xd3, w, wd, 1e-5), a.steps, a.warmup)
        by = 8 * 4096 * 1024 * x3.element_size() * 4  # read x, x_dot; write y, y_dot
        print(json.dumps({"metric": "RMSNorm JVP [8,4096,1024]", "value": by / ms / 1e6, "unit": "GB/s",
                          "dtype": dt_name, "ms": ms,
                          "roofline": {"bound": "hbm", "achieved": by / ms / 1e6, "peak": hbm,
                                       "frac": by / ms / 1e6 / hbm}}), flush=True)


def zipf_ids(n, vocab, seed, s=1.1):
    g = torch.Generator().manual_seed(seed)
    ranks = torch.arange(1, vocab + 1, dtype=torch.float64)
    pmf = ranks.pow(-s)
    cdf = torch.cumsum(pmf / pmf.sum(), 0)
    return torch.searchsorted(cdf, torch.rand(n, generator=g, dtype=torch.float64)).clamp_(max=vocab - 1)


PROF_NAMES = {0: "ssm_chunk_fwd", 1: "ssm_compose", 2: "ssm_out_fwd", 3: "ssm_chunk_bwd",
              4: "ssm_main_bwd", 5: "gemm_tc", 6: "gemm_simt", 7: "rmsnorm_fwd", 8: "rmsnorm_bwd",
              9: "embedding", 10: "ce", 11: "adamw"}


def run_gpu(a, rank, world, local_rank):
    from icml_b200 import _lib

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    pg = None
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=dev)
        pg = torch.distributed.group.WORLD
    L = _lib.lib()
    r = _measure_model(a, rank, world, local_rank, dev, pg, L)
    line = None
    if rank == 0:
        line = _line_of(a, world, r)
        if world == 1 and not a.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(a)
    # the model of the benchmark configurations (Mamba-standard block) on the same sequence, when the
    # headline runs the reference's own SSM variant
    if a.variant == "reference" and not a.no_std_companion:
        b = argparse.Namespace(**vars(a))
        b.variant = "std"
        try:
            r2 = _measure_model(b, rank, world, local_rank, dev, pg, L)
            if rank == 0:
                l2 = _line_of(b, world, r2)
                line["mamba_standard"] = {k: l2[k] for k in ("metric", "value", "unit", "ms_per_step", "scaling",
                                                             "config", "peak_hbm_gb", "clocks", "e2e",
                                                             "gpu_launches", "cuda_graph", "kernels",
                                                             "dominant_kernel", "roofline")}
        except Exception as e:  # the headline line is printed whatever happens to the companion
            if rank == 0:
                line["mamba_standard"] = {"error": f"{type(e).__name__}: {e}"[:300]}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if pg is not None:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def _measure_model(a, rank, world, local_rank, dev, pg, L):
    """Build the LM of `a`, run its warm-up, profiled, timed and end-to-end steps; returns the
    measurements (max over ranks) and releases the model's graph and memory."""
    import ctypes
    from icml_b200.lm import PGFLanguageModel

    act = torch.bfloat16 if a.dtype == "bf16" else torch.float32
    torch.manual_seed(1234)
    if a.variant == "std":
        model = PGFLanguageModel(a.vocab, a.d_model, 16, a.d_ff, a.layers, a.block_size, dev, act_dtype=act,
                                 variant="std", tie_embeddings=True, final_norm=True, expand=2, d_conv=4,
                                 dt_rank=a.dt_rank, stash=a.stash)
    else:
        model = PGFLanguageModel(a.vocab, a.d_model, 16, a.d_ff, a.layers, a.block_size, dev, act_dtype=act,
                                 stash=a.stash)
    for p in model.params:  # identical replicas
        if pg is not None:
            torch.distributed.broadcast(p.data, 0)

    Lr = per_rank_len(a, world)
    if world > 1 and a.parallel == "sp":
        # the one sequence; this rank holds the segment [rank*Lr, (rank+1)*Lr)
        full = zipf_ids(a.batch * (a.seq_len + 1), a.vocab, seed=100).reshape(a.batch, -1)
        ids_host = full[:, rank * Lr: (rank + 1) * Lr + 1]
    else:
        ids_host = zipf_ids(a.batch * (Lr + 1), a.vocab, seed=100 + rank).reshape(a.batch, Lr + 1)
    inp_host = ids_host[:, :-1].contiguous().pin_memory()
    tgt_host = ids_host[:, 1:].contiguous().pin_memory()
    inp = inp_host.to(dev)
    tgt = tgt_host.to(dev)

    flat_opt = getattr(model, "optimizer_kind", "torch") == "flat"

    def allreduce_grads():
        if pg is None:
            return False
        grads = [p.grad for p in model.params]
        flat = torch.cat([g.reshape(-1) for g in grads])
        torch.distributed.all_reduce(flat)
        flat.div_(world)
        o = 0
        for g in grads:
            n = g.numel()
            g.copy_(flat[o:o + n].view_as(g))
            o += n
        return False

    from icml_b200 import seqpar
    sp = seqpar.SeqGroup.from_default() if (world > 1 and a.parallel == "sp") else None
    # N GPUs: each layer's gradients are all-reduced (in the flat optimizer buffer, on a side stream)
    # as soon as its backward returns, overlapping the backward of the layers below
    reducer = None
    if pg is not None and flat_opt:
        from icml_b200.optim import OverlappedGradReduce
        RO = torch.distributed.ReduceOp
        reducer = OverlappedGradReduce(model, RO.SUM if sp is not None else RO.AVG)

    def step(x, y):
        model.optimizer.zero_grad(set_to_none=True)
        if sp is not None:
            loss, grads = seqpar.lm_forward_backward(model, x, y, sp, reducer=reducer)
            if reducer is not None:
                model.optimizer.step(gather=False)
                return loss
            model._assign(grads)  # gradients already summed
        elif reducer is not None:
            loss, grads = model.forward_backward(x, y, on_layer_grads=reducer.layer)
            reducer.finish(grads)
            model.optimizer.step(gather=False)
            return loss
        else:
            loss, grads = model.forward_backward(x, y)
            model._assign(grads)
            allreduce_grads()
        model.optimizer.step()
        return loss

    for _ in range(a.warmup):
        step(inp, tgt)
    torch.cuda.synchronize()

    def barrier():
        if pg is not None:
            torch.distributed.barrier()

    # ---------------- per-kernel breakdown: eager steps with libpgf's CUDA-event timers
    n_prof = min(a.steps, 3)
    barrier()
    torch.cuda.synchronize()
    # peak HBM of a step: measured on these eager steps (a graph replay reuses the memory pool its
    # capture allocated, so the allocator sees no new peak during replays)
    torch.cuda.reset_peak_memory_stats(dev)
    n0 = L.pgf_launch_count()
    L.pgf_profile(1)
    for _ in range(n_prof):
        step(inp, tgt)
    torch.cuda.synchronize()
    L.pgf_profile(0)
    launches_eager = (L.pgf_launch_count() - n0) // n_prof
    peak_gb = torch.cuda.max_memory_allocated(dev) / 1e9
    prof_ms, prof_n, prof_w = {}, {}, {}
    for i, nm in PROF_NAMES.items():
        c = ctypes.c_longlong(0)
        t = ctypes.c_double(0.0)
        w = ctypes.c_double(0.0)
        L.pgf_profile_read(i, ctypes.byref(c), ctypes.byref(t), ctypes.byref(w))
        if c.value:
            prof_n[nm] = c.value / n_prof
            prof_ms[nm] = t.value / n_prof
            prof_w[nm] = w.value / n_prof

    # ---------------- the step (with its collectives on N GPUs) as one CUDA graph
    graphed = None
    if not a.no_graph:
        from icml_b200.lm import GraphedStep
        barrier()
        err = None
        try:
            graphed = GraphedStep(step, inp, tgt, warmup=1)
        except Exception as e:  # capture refused: every rank falls back to eager launches together
            err = e
            graphed = None
        ok = torch.tensor([0 if err else 1], device=dev, dtype=torch.int32)
        if pg is not None:
            torch.distributed.all_reduce(ok, op=torch.distributed.ReduceOp.MIN)
        if int(ok.item()) == 0:
            if graphed is not None:
                graphed.release()
                graphed = None
            if rank == 0:
                print(f"[bench] CUDA-graph capture unavailable ({err}); timing eager launches", file=sys.stderr)
        barrier()
    if graphed is not None:
        run_step = lambda x, y: graphed.run(x, y)  # noqa: E731
        launches = graphed.launches
    else:
        run_step = step
        launches = launches_eager

    # ---------------- device-timed region: inputs resident in HBM
    sampler = ClockSampler(local_rank)
    sampler.start()
    time.sleep(0.3)
    barrier()
    torch.cuda.synchronize()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(a.steps):
        loss = run_step(inp, tgt) if graphed is None else graphed.run()
    ev1.record()
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop()
    ms = ev0.elapsed_time(ev1)
    t_all = torch.tensor([ms], device=dev)
    if pg is not None:
        torch.distributed.all_reduce(t_all, op=torch.distributed.ReduceOp.MAX)
    ms = t_all.item()
    ms_step = ms / a.steps
    tokens = a.batch * Lr * world * a.steps
    value = tokens / (ms / 1e3)

    # ---------------- end to end: host ids -> device each step, loss read back each step
    barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.steps):
        if graphed is None:
            x = inp_host.to(dev, non_blocking=True)
            y = tgt_host.to(dev, non_blocking=True)
            loss = step(x, y)
        else:
            loss = graphed.run(inp_host, tgt_host)  # copies from pinned host memory into the graph's inputs
        loss_val = loss.item()
    e1.record()
    torch.cuda.synchronize()
    barrier()
    te = torch.tensor([e0.elapsed_time(e1)], device=dev)
    if pg is not None:
        torch.distributed.all_reduce(te, op=torch.distributed.ReduceOp.MAX)
    e2e = tokens / (te.item() / 1e3)

    r = {"value": value, "ms_step": ms_step, "e2e": e2e, "peak_gb": peak_gb, "clocks": clocks,
         "launches": launches, "graphed": graphed is not None, "loss": loss_val,
         "prof_ms": prof_ms, "prof_n": prof_n, "prof_w": prof_w, "h2d": inp_host.numel() * 8 * 2}
    if graphed is not None:
        torch.cuda.synchronize()
        graphed.release()  # the graph holds NCCL work on N GPUs: release it before the process group
        del graphed
    del model, reducer, inp, tgt
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return r


def _line_of(a, world, r):
    """The JSON line of one measured model (rank 0)."""
    prof_ms, prof_n, prof_w, ms_step = r["prof_ms"], r["prof_n"], r["prof_w"], r["ms_step"]
    dom = max(prof_ms, key=prof_ms.get) if prof_ms else None
    # per-kernel figures come from the eager profiled steps (graph replays carry no timers)
    traffic = TRAFFIC_DEFAULT if default_workload(a, world) else {}
    kernels = {k: {"launches_per_step": prof_n[k], "ms_per_step": prof_ms[k],
                   "share_of_step": prof_ms[k] / ms_step if ms_step else None,
                   "roofline": roofline_entry(k, prof_ms[k], prof_n[k], prof_w[k], traffic.get(k))}
               for k in prof_ms}
    clocks = r["clocks"]
    compute_roofline = None
    if "ssm_main_bwd" in kernels and default_workload(a, world):
        mhz = clocks.get("sm_mhz") or clocks.get("sm_max_mhz") or 1965.0
        compute_roofline = issue_roofline(kernels["ssm_main_bwd"]["roofline"]["ms_per_launch"], mhz)
    return {
        "metric": metric_of(a), "value": r["value"], "unit": UNIT, "n_gpus": world, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": scaling_of(a, world),
        "vs_baseline": None, "dtype": a.dtype, "data": "synthetic (Zipf 1.1 token ids, random init)",
        "config": dict(config_of(a, world), launch=(
            "whole step (with its collectives) captured once as a CUDA graph, replayed each step"
            if r["graphed"] else "eager launches")), "impl": "b200",
        "peak_hbm_gb": r["peak_gb"], "loss": r["loss"], "clocks": clocks,
        "e2e": {"value": r["e2e"], "unit": UNIT, "h2d_bytes_per_step": r["h2d"], "d2h_bytes_per_step": 4},
        "gpu_launches": int(r["launches"]),
        "cuda_graph": r["graphed"],
        "kernels": kernels, "dominant_kernel": dom,
        "roofline": kernels[dom]["roofline"] if dom else None,
        "compute_roofline": compute_roofline,
    }


if __name__ == "__main__":
    main()
