"""Benchmark of the quantized decode path on B200: decode tok/s and % of the HBM roofline.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config internlm-q4-1792]

Default workload (BASELINE config 3 at its headline point): InternLM2.5-1.8B-shaped decoder, random-init (seed 2,
N(0, 0.02) weights, 4-bit affine group 64 with fp16 scale/bias), batch 1, a history of 1,792 - W positions (the KV
cache rows filled on the device with seeded N(0, 1) fp16 values: throughput does not depend on their content), W
warm-up steps, then K greedy decode steps at positions 1,792 .. 1,792+K-1. A step is one token: one CUDA-graph replay
of the step's 121 kernels (AGXC_FUSED=1 in the environment: the fused persistent step kernel instead; the line's
"fused_step" block times it beside the default either way). Inputs are far larger than L2 (0.96 GB of packs + 0.18 GB
of KV per token against a 126 MB L2), so no flush is needed between steps.

    python bench.py --kernel-case ffn|qkv|wo|down|head|attn [--case-batch B]
        one launch of that kernel of the workload (after 3 warm-ups) through the C-ABI: the ncu capture case
        (B >= 32: the batched tensor-core GEMM agxc_qmm on the kernel's shape)

    python bench.py --trace-step [--config ...]
        one traced decode step of a batch-1 workload (AGXC_OPT_TRACE: every CTA's entry, dependency-wait, staging,
        first-chunk, loop-end and exit times on the global timer), printed as per-phase means over the middle layers

One JSON line on rank 0:
  value          tokens/s over the K timed steps (device time, CUDA events, inputs resident in HBM), summed over ranks
  e2e            the same steps through the public C-ABI decode call with a host->device copy of each step's input
                 token (pinned) and a device->host read of its chosen token every step, the host waiting for step
                 i - 1 once step i is queued (sync_each 2, a streaming server's loop); "lockstep" = the same with the
                 host waiting for every step before queueing the next (sync_each 1)
  roofline       the dominant kernel (largest share of step time, from a CUDA-event profile of every launch):
                 algorithmic bytes per launch / its mean launch time, against the measured HBM copy bandwidth
  step_roofline  the whole step: (pack bytes + KV bytes read) per token x tokens/s, against the same peak
  cpu_baseline   the reference's CPU decode step (its QSim chain) as the numpy FP32 port in oracle/cpu_decode.py,
                 timed on this host's cores on a bounded sample (--cpu-tokens whole tokens: every layer, the head and
                 the argmax)
  prefill        the same model's prefill section on a prompt of `history` tokens (device time, prompt tok/s)
Multi-GPU (torchrun, --gpus N): configs 1-4 do not shard (replicas only): every rank decodes its own sequence on its
own GPU, timing is the max over ranks, `value` sums the tokens of all ranks ("scaling": "weak").

Other workloads (--config):
  internlm-q{4,8}-1792-b{32,128}   batch 32 / 128 sequences: the tensor-core GEMM decode step
  internlm7b-q4-8192-b64-tp        BASELINE config 5: the 7B shape, 64 sequences x 8,192-token histories, tensor
                                   parallel over the N ranks ("scaling": "strong"); --tp-allreduce fused | nccl
  minilm-b32-s128                  BASELINE config 2: the MiniLM-L6 sentence encoder, 32 x 128 tokens, sentences/s
                                   against the tensor-core roofline, L2 flushed before every timed forward
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

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CONFIGS = {
    # name: (model, bits, batch, history)
    "internlm-q4-1792": ("internlm2.5-1.8b", 4, 1, 1792),
    "internlm-q4-196": ("internlm2.5-1.8b", 4, 1, 196),
    "internlm-q8-1792": ("internlm2.5-1.8b", 8, 1, 1792),
    "internlm-q8-1792-b8": ("internlm2.5-1.8b", 8, 8, 1792),
    "internlm-q4-1792-b32": ("internlm2.5-1.8b", 4, 32, 1792),     # tensor-core GEMM step (batch >= 32)
    "internlm-q4-1792-b128": ("internlm2.5-1.8b", 4, 128, 1792),
    "internlm-q8-1792-b32": ("internlm2.5-1.8b", 8, 32, 1792),
    "internlm-q8-1792-b128": ("internlm2.5-1.8b", 8, 128, 1792),
    # tensor parallel over all ranks (--gpus N = TP N; strong scaling: the same 64 sequences at every N)
    "internlm7b-q4-8192-b64-tp": ("internlm2.5-7b", 4, 64, 8192),
    "qwen-q4-196": ("qwen2.5-0.5b", 4, 1, 196),
}
METRIC = "decode tok/s and % HBM roofline (batch 1, ctx 1792, 4-bit) vs CPU ref"
TP_CONFIGS = {"internlm7b-q4-8192-b64-tp"}
# the MiniLM-L6 sentence encoder, 32 sequences x 128 tokens, valid lengths uniform in 16..128
ENCODER_CONFIGS = {"minilm-b32-s128": (32, 128)}
ENCODER_METRIC = "encoder sentences/s (MiniLM-L6, batch 32 x seq 128, fp16 tensor cores) vs CPU ref"
KIND_NAMES = ["qkv", "attn", "wo", "ffn", "down", "head"]


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class Clocks:
    """SM clock, max SM clock and throttle reasons sampled DURING the timed region, every 5 ms, by a host thread through
    NVML (read-only queries; the device is found by the CUDA device's UUID, so CUDA_VISIBLE_DEVICES cannot point it
    at another GPU). Each sample carries its own wall time and is kept when it falls inside the timed region. Without
    NVML: nvidia-smi, line-buffered, its samples placed by their own timestamps."""
    NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
    # NVML clock-event reason bits (nvml.h): HwSlowdown, HwThermalSlowdown, SwThermalSlowdown, SwPowerCap
    BITS = [0x8, 0x40, 0x20, 0x4]
    Q = ("timestamp,clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.samples = []          # (wall time, sm MHz, max sm MHz, [reason names])
        self.t0 = self.t1 = None
        self.proc = None
        self.source = None
        self._stop = threading.Event()

    def _uuid(self):
        import torch
        u = str(torch.cuda.get_device_properties(self.index).uuid)
        return u if u.startswith("GPU-") else "GPU-" + u

    def start(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByUUID(self._uuid())
            mx = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
            reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                pynvml.nvmlDeviceGetCurrentClocksThrottleReasons

            def run():
                while not self._stop.is_set():
                    t = time.time()
                    sm = float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM))
                    r = int(reasons(h))
                    self.samples.append((t, sm, mx, [n for n, bit in zip(self.NAMES, self.BITS) if r & bit]))
                    time.sleep(0.005)
            self.source = "nvml"
        except Exception:  # noqa: BLE001 - fall back to nvidia-smi
            try:
                self.proc = subprocess.Popen(["stdbuf", "-oL", "nvidia-smi", "-i", self._uuid(),
                                              "--query-gpu=" + self.Q, "--format=csv,noheader,nounits", "-lms", "20"],
                                             stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            except Exception:  # noqa: BLE001
                return self

            def run():
                for line in self.proc.stdout:
                    parts = [x.strip() for x in line.split(",")]
                    try:
                        t = time.mktime(time.strptime(parts[0].split(".")[0], "%Y/%m/%d %H:%M:%S"))
                        t += float("0." + parts[0].split(".")[1]) if "." in parts[0] else 0.0
                        self.samples.append((t, float(parts[1]), float(parts[2]),
                                             [n for n, v in zip(self.NAMES, parts[3:7]) if v.lower() == "active"]))
                    except (ValueError, IndexError):
                        continue
            self.source = "nvidia-smi"
        self.thread = threading.Thread(target=run, daemon=True)
        self.thread.start()
        t_end = time.time() + 3.0
        while not self.samples and time.time() < t_end:  # the sampler is up before the timed region starts
            time.sleep(0.005)
        return self

    def mark_start(self):
        self.t0 = time.time()

    def mark_end(self):
        self.t1 = time.time()

    def stop(self):
        self._stop.set()
        if self.proc:
            time.sleep(0.1)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:  # noqa: BLE001
                self.proc.kill()
        if getattr(self, "thread", None) is not None:
            self.thread.join(timeout=2)

    def summary(self):
        inside = [x for x in list(self.samples) if self.t0 is not None and self.t0 <= x[0] <= self.t1]
        if not inside:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0,
                    "source": self.source}
        reasons = sorted({n for x in inside for n in x[3]})
        return {"sm_mhz": statistics.median(x[1] for x in inside), "sm_max_mhz": max(x[2] for x in inside),
                "reasons": reasons, "samples": len(inside), "source": self.source}


def dist_setup(gpus):
    if gpus <= 1 or "RANK" not in os.environ:
        return 0, 1, 0, None
    import datetime

    import torch
    import torch.distributed as dist
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    return rank, world, local, dist


def cpu_baseline_sample(m, tokens, pos):
    """Time the numpy FP32 port of the reference's CPU decode step (oracle/cpu_decode.py) on `tokens` whole tokens
    (every layer, the head, the first argmax) at positions pos .., over this model's packs copied to the host."""
    from oracle.cpu_decode import CpuDecoder
    cpu = CpuDecoder(m.shape, m.packs, m.bits, m.cfg["scale_dtype"], pos + tokens + 2)
    cpu.fill_history(pos, seed=1792)
    tok = 1
    t0 = time.perf_counter()
    for i in range(tokens):
        tok = cpu.decode_token(tok, pos + i)
    return (time.perf_counter() - t0) / tokens, cpu.threads


def sm_max_mhz():
    """The device's maximum SM clock (NVML), to turn the cycle profile into time; 1965 (B200) without NVML."""
    try:
        import pynvml
        import torch
        pynvml.nvmlInit()
        u = str(torch.cuda.get_device_properties(0).uuid)
        h = pynvml.nvmlDeviceGetHandleByUUID(u if u.startswith("GPU-") else "GPU-" + u)
        return float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
    except Exception:  # noqa: BLE001
        return 1965.0


def trace_fused_step(args, m, hist):
    """--trace-step on the fused step: one traced step's per-CTA marks reduced to per-phase times (µs), means over
    layers 2 .. L-2. Per layer: qkv = its slowest CTA's qkv work after x was complete; attn_wait = from the last qkv
    tile to the last attention CTA passing its group's dependency; attn = attention work (slowest CTA); o_wait / o_proj
    = the same for the merge + o_proj; h_wait = to the last CTA passing the h dependency; ffn = the FFN work (slowest
    CTA); x_wait = from the last FFN unit to the last CTA passing the next layer's x dependency; layer = x-complete to
    x-complete. `timeline`: every mark of the layer (assemble.DecodeModel.trace_fused) as [median, max] over the CTAs
    that reach it, µs after the layer's x-complete (the producer's marks may precede it: negative). `profile_us`:
    the cycle profile (assemble.DecodeModel.profile_fused), µs of the whole step per region for the median CTA."""
    from agxforge.inference.assemble import FUSED_TRACE_MARKS as NM
    names = ["q_dep", "q_done", "a_dep", "a_done", "o_dep", "o_done", "f_dep", "f_done", "q_normed", "q_tile1",
             "a_keys", "o_merged", "f_normed", "f_gu1", "f_gu", "f_down1", "p_q", "p_a", "p_f", "p_f_last",
             "q_landed", "q_t0done", "f_gu1_landed", "f_gu1_t0done", "f_gu2_landed", "p_down"]
    m.start(0, [1])
    m.fill_history(0, hist - args.warmup, seed=1792)
    m.decode(args.warmup, want_tokens=False)
    m.set_option("trace", 1)
    m.decode(1, want_tokens=False)
    tr = m.trace_fused().astype(np.float64)
    prof = m.profile_fused()
    m.close()
    L = (tr.shape[0] - 2) // NM
    rec, tl = [], []
    for l in range(2, L - 2):
        b = NM * l
        mx = lambda k: tr[b + k][tr[b + k] > 0].max()   # noqa: E731
        mn = lambda k: tr[b + k][tr[b + k] > 0].min()   # noqa: E731
        nxt = tr[b + NM][tr[b + NM] > 0].max()
        rec.append(dict(qkv=mx(1) - mx(0), attn_wait=mx(2) - mx(1), attn=mx(3) - mx(2), o_wait=mx(4) - mx(3),
                        o_proj=mx(5) - mx(4), h_wait=mx(6) - mx(5), ffn=mx(7) - mx(6), x_wait=nxt - mx(7),
                        layer=nxt - mx(0), x_skew=mx(0) - mn(0)))
        t0 = mx(0)
        row = {}
        for k, nm in enumerate(names):
            v = tr[b + k][tr[b + k] > 0] - t0
            row[nm] = (float(np.median(v)), float(v.max())) if v.size else (np.nan, np.nan)
        tl.append(row)
    phases = {k: round(float(np.mean([r[k] for r in rec])) / 1e3, 2) for k in rec[0]}
    timeline = {nm: [round(float(np.nanmean([r[nm][0] for r in tl])) / 1e3, 2),
                     round(float(np.nanmean([r[nm][1] for r in tl])) / 1e3, 2)] for nm in names}
    head = tr[NM * L + 1][tr[NM * L + 1] > 0].max() - tr[NM * L][tr[NM * L] > 0].max()
    step = tr[NM * L + 1][tr[NM * L + 1] > 0].max() - tr[0][tr[0] > 0].min()
    mhz = sm_max_mhz()
    profile = {k: round(float(np.median(v)) / mhz, 1) for k, v in prof.items()}   # µs over the step, median CTA
    print(json.dumps(dict(trace_step=args.config, fused=True, layers=L, step_us=round(step / 1e3, 1),
                          head_us=round(head / 1e3, 2), phases=phases, timeline=timeline,
                          profile_us=profile, profile_mhz=mhz)), flush=True)


def trace_step(args):
    """--trace-step: one traced step of a batch-1 config after the bench's warm-up, reduced to per-phase means (µs)
    over layers 2 .. L-2. For phase i: handoff = its last CTA past the dependency wait - phase i-1's last exit;
    stage = activations staged - wait; first = first weight chunk landed - staged; loop = last chunk consumed - first
    chunk; total = its last exit - phase i-1's last exit (all taken at the slowest CTA)."""
    import numpy as np
    from agxforge.inference import assemble
    model, bits, batch, hist = CONFIGS[args.config]
    if batch != 1:
        raise SystemExit("--trace-step: batch-1 configs only")
    m = assemble.build(dict(model=model, bits=bits, batch=1, cap=hist + 16, seed=2))
    if m.fused:
        trace_fused_step(args, m, hist)
        return
    m.start(0, [1])
    m.fill_history(0, hist - args.warmup, seed=1792)
    m.decode(args.warmup, want_tokens=False)
    m.set_option("trace", 1)
    m.decode(1, want_tokens=False)
    m.trace()                                  # the first traced step primes the trace buffers
    m.decode(1, want_tokens=False)
    tr = m.trace()
    m.close()
    L = len(tr) // 5
    per = {}
    for i in range(10, 5 * (L - 2)):
        d, p = tr[i], tr[i - 1]
        rec = dict(handoff=d["wait"][1] - p["exit"][1], total=d["exit"][1] - p["exit"][1],
                   entry_spread=d["entry"][1] - d["entry"][0], exit_spread=d["exit"][1] - d["exit"][0])
        if "staged" in d:
            rec.update(stage=d["staged"][1] - d["wait"][1], first=d["landed"][1] - d["staged"][1],
                       loop=d["looped"][1] - d["landed"][1])
        per.setdefault(d["kind"], []).append(rec)
    phases = {k: {f: round(float(np.mean([r[f] for r in v])) / 1e3, 2) for f in v[0]} for k, v in per.items()}
    head = tr[-1]
    print(json.dumps(dict(trace_step=args.config, layers=L, step_us=round((head["exit"][1] - tr[0]["entry"][0]) / 1e3, 1),
                          head_us=round((head["exit"][1] - tr[-2]["exit"][1]) / 1e3, 2), phases=phases)), flush=True)


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for ln in f:
                if ln.startswith("model name"):
                    return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def workload_config(args, world, model, bits, batch, hist, tp):
    """The config object of a decode workload's line: identical in both arms (--impl ours / reference)."""
    K = args.steps
    step_bytes = None
    try:
        from agxforge.inference import models
        S = models.get(model)
        step_bytes = S.weight_bytes(bits) + batch * S.kv_bytes_per_position() * (hist + (K - 1) / 2.0 + 1)
    except Exception:  # noqa: BLE001
        pass
    return dict(workload=args.config, model=model, bits=bits, group=64, scale_dtype="fp16", batch=batch,
                history=hist, positions=[hist, hist + K - 1],
                parallelism=("tp%d" % tp) if tp > 1 else ("replicas" if world > 1 else "1gpu"),
                l2="inputs larger than L2 (%.2f GB per step vs 126 MB L2)" % (step_bytes / 1e9) if step_bytes
                else "inputs larger than L2")


def run_reference(args, rank, world):
    """--impl reference: the reference's CPU implementation of the path on this host's cores, with the same config,
    metric and unit as our arm. The reference's own CPU references (its Python package) do not travel with this
    repository, so the timed code is their restatement, oracle/cpu_decode.py (the QSim chain as numpy FP32, row
    blocks on a thread pool over every core). Nothing here loads the CUDA library: the packs are made on the host from
    the config's seed (N(0, 0.02) weights quantised by oracle.pack, the reference's quantize). Each step is one whole
    token (every layer, the head, the first argmax) at the positions our arm times: W warm-up tokens at hist - W ..
    hist - 1 over a seeded history, then K timed tokens at hist .. hist + K - 1."""
    from agxforge.inference import models       # shapes only (plain Python)
    from oracle import cpu_decode as CD
    model, bits, batch, hist = CONFIGS[args.config]
    tp = world if args.config in TP_CONFIGS else 1
    S = models.get(model)
    K, W = args.steps, args.warmup
    t0 = time.perf_counter()
    packs = CD.host_packs(S, bits, "fp16", 2)
    pack_s = time.perf_counter() - t0
    cpu = CD.CpuDecoder(S, packs, bits, "fp16", hist + K + 2)
    cpu.fill_history(hist - W, seed=1792)
    tok = 1
    for i in range(W):
        tok = cpu.decode_token(tok, hist - W + i)
    t0 = time.perf_counter()
    for i in range(K):
        tok = cpu.decode_token(tok, hist + i)
    dt = time.perf_counter() - t0
    per_token = dt / K
    v = batch / per_token if batch > 1 else 1.0 / per_token
    cores = cpu.threads
    sample = ("%d whole tokens (all %d layers, head, argmax) at positions %d..%d over a seeded %d-position history, "
              "batch %d of %d sequences (the CPU step is per sequence)" % (K, S.LAYERS, hist, hist + K - 1, hist - W,
                                                                             1, batch))
    line = dict(metric=METRIC, impl="reference", value=round(1.0 / per_token, 5), unit="tok/s", n_gpus=world,
                steps=K, warmup=W, ms_per_step=round(per_token * 1e3, 1), higher_is_better=True,
                scaling="strong" if tp > 1 else "weak", vs_baseline=None, dtype="f32", data="synthetic",
                config=workload_config(args, world, model, bits, batch, hist, tp),
                cpu_baseline=dict(value=round(1.0 / per_token, 5), unit="tok/s", cores=cores, cpu=cpu_model(),
                                  kind="port", sample=sample, packs_made_on_host_s=round(pack_s, 1)),
                e2e=dict(value=round(1.0 / per_token, 5), unit="tok/s", h2d_bytes_per_step=0, d2h_bytes_per_step=0))
    del v
    print(json.dumps(line), flush=True)


def encoder_inputs(B, S, seed, vocab=30522):
    """Config 2's inputs: uniform-random ids, per-row valid lengths uniform in 16..S, 0/1 masks."""
    rng = np.random.default_rng(seed)
    ids = rng.integers(0, vocab, (B, S)).astype(np.int32)
    lens = rng.integers(16, S + 1, B)
    return ids, (np.arange(S)[None, :] < lens[:, None]).astype(np.int32)


def encoder_cpu_sample(B, S, sample):
    """The reference's CPU encoder (graph_reference's FP64 policy, restated in oracle/encoder.py) on `sample` of the
    B sequences, all host threads: seconds per sentence."""
    from oracle import encoder as E
    params = E.make_params(1)
    ids, mask = encoder_inputs(B, S, 1)
    t0 = time.perf_counter()
    E.forward(params, ids[:sample], mask[:sample], policy="fp64")
    return (time.perf_counter() - t0) / sample, os.cpu_count()


def run_encoder_reference(args):
    B, S = ENCODER_CONFIGS[args.config]
    per = [encoder_cpu_sample(B, S, 4)[0] for _ in range(max(1, args.ref_steps))]
    v = 1.0 / statistics.median(per)
    cores = os.cpu_count()
    line = dict(metric=ENCODER_METRIC, impl="reference", value=round(v, 3), unit="sentences/s", n_gpus=args.gpus,
                steps=args.steps, warmup=args.warmup, ms_per_step=round(B * 1e3 / v, 1), higher_is_better=True,
                scaling="weak", vs_baseline=None, dtype="f64", data="synthetic",
                config=dict(workload=args.config, model="minilm-l6", batch=B, seq=S),
                cpu_baseline=dict(value=round(v, 3), unit="sentences/s", cores=cores, kind="port",
                                  sample="4 of the %d sequences of one batch, FP64 graph reference, median of %d"
                                         % (B, len(per))),
                e2e=dict(value=round(v, 3), unit="sentences/s", h2d_bytes_per_step=0, d2h_bytes_per_step=0))
    print(json.dumps(line), flush=True)


def run_encoder(args, rank, world, local, dist):
    """Config 2 on each GPU (replicas only: the encoder's batches are independent)."""
    import torch
    from agxforge.inference.encoder import MINILM_L6, Encoder
    B, S = ENCODER_CONFIGS[args.config]
    K, W = args.steps, args.warmup
    enc = Encoder.synthetic(MINILM_L6, seed=1 + rank, max_batch=B, max_seq=S, device=local)
    ids, mask = encoder_inputs(B, S, 1 + rank)
    inputs = dict(token_ids=ids, attention_mask=mask)
    for _ in range(W):
        enc.forward(inputs)
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    clk = Clocks(local).start()
    clk.mark_start()
    t = enc.replay(K, flush_l2=True)       # K forwards, inputs resident, L2 flushed before each, device time
    clk.mark_end()
    clk.stop()
    gpu_ms = t["gpu_ms"]
    # e2e: the public forward call, host ids/mask in and embeddings out every batch
    t0 = time.perf_counter()
    for _ in range(K):
        enc.forward(inputs)
    e2e_s = time.perf_counter() - t0
    if dist is not None:
        tt = torch.tensor([gpu_ms, e2e_s], device="cuda")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        gpu_ms, e2e_s = float(tt[0].item()), float(tt[1].item())
    value = world * B * K / (gpu_ms / 1e3)
    e2e_v = world * B * K / e2e_s
    prof = enc.profile(B, S, reps=3)
    W_, F_, M = 384, 1536, B * S
    flops = {"qkv": 2 * M * 3 * W_ * W_, "o_proj": 2 * M * W_ * W_, "ffn_up": 2 * M * F_ * W_,
             "ffn_down": 2 * M * W_ * F_}
    dom = max(flops, key=lambda k: prof[k]["ms"])
    per_launch_ms = prof[dom]["ms"] / max(1, prof[dom]["launches"])
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peak, src = float(json.load(f)["bf16_tflops"]), "measured (bf16 burst)"
    except Exception:
        peak, src = 1590.0, "fallback"
    achieved = flops[dom] / (per_launch_ms / 1e3) / 1e12
    total_flops = 6 * sum(flops.values()) + 6 * 4 * B * 12 * S * S * 32
    cpu = None
    if rank == 0 and not args.no_cpu:
        per, cores = encoder_cpu_sample(B, S, 4)
        cpu = dict(value=round(1.0 / per, 3), unit="sentences/s", cores=cores, kind="port",
                   sample="4 of the %d sequences of one batch, FP64 graph reference (oracle/encoder.py)" % B)
    if rank == 0:
        line = dict(
            metric=ENCODER_METRIC, value=round(value, 1), unit="sentences/s", n_gpus=world, steps=K, warmup=W,
            ms_per_step=round(gpu_ms / K, 4), higher_is_better=True, scaling="weak", vs_baseline=None, dtype="f16",
            data="synthetic (seeded random-init parameters, uniform-random ids, valid lengths 16..128)",
            config=dict(workload=args.config, model="minilm-l6", batch=B, seq=S,
                        parallelism="replicas" if world > 1 else "1gpu",
                        l2="L2 flushed (256 MB written) before every timed forward; the working set (21 MB of "
                           "weights + activations) would otherwise stay in the 126 MB L2"),
            e2e=dict(value=round(e2e_v, 1), unit="sentences/s", h2d_bytes_per_step=2 * B * S * 4,
                     d2h_bytes_per_step=B * W_ * 4),
            roofline=dict(bound="tensor", kernel=dom, achieved=round(achieved, 1), peak=peak, unit="TFLOP/s",
                          frac=round(achieved / peak, 4), traffic=None, peak_source=src,
                          flops_per_launch=flops[dom], us_per_launch=round(per_launch_ms * 1e3, 2)),
            step_roofline=dict(bound="tensor", achieved=round(total_flops / (gpu_ms / K / 1e3) / 1e12, 1), peak=peak,
                               unit="TFLOP/s", frac=round(total_flops / (gpu_ms / K / 1e3) / 1e12 / peak, 4),
                               flops_per_step=total_flops),
            kernels={k: dict(ms=round(v["ms"] / 3, 4), launches=v["launches"] // 3) for k, v in prof.items()},
            cpu_baseline=cpu, clocks=clk.summary(), gpu_launches=int(t["launches"] * K))
        print(json.dumps(line), flush=True)
    enc.close()


def kernel_case(args, rank):
    """One launch of one kernel of the workload, after 3 warm-up launches of it (the ncu capture case: `-k` on the
    kernel's name, `-s 3 -c 1`). GEMV kernels run through agxc_qmv on packs of the workload's shape (same planner and
    kernels as the model); attention through agxc_attention_dev on a cache of the workload's shape at position 1,792."""
    import torch
    from agxforge.kernels import attention as A
    from agxforge.kernels import qmv as Q
    from agxforge.inference import models
    model, bits, batch, hist = CONFIGS[args.config]
    S = models.get(model)
    torch.manual_seed(5)
    if args.kernel_case == "attn":
        cap = hist + 8
        K = torch.randn(batch, S.KV_HEADS, cap, S.HEAD_DIM, device="cuda").half()
        V = torch.randn(batch, S.KV_HEADS, cap, S.HEAD_DIM, device="cuda").half()
        q = (torch.randn(batch, S.HEADS, S.HEAD_DIM, device="cuda") * 0.1).half()
        for _ in range(4):
            A.attention(q, K, V, [hist] * batch)
    elif (args.case_batch or batch) >= 32:
        # the batched tensor-core GEMM (agxc_qmm) on the kernel's shape (gate/up as one plain 2F-row pack)
        from agxforge.kernels.qmm import qmm
        B = args.case_batch or batch
        shapes = {r: (n, k) for r, n, k in S.matrices()}
        n, k = {"qkv": shapes["qkv"], "wo": shapes["wo"], "ffn": (2 * shapes["gate"][0], shapes["gate"][1]),
                "down": shapes["down"], "head": (S.VOCAB, S.D_MODEL)}[args.kernel_case]
        W = torch.randn(n, k, device="cuda") * 0.02
        pk = Q.Pack(*Q.quantize(W, bits=bits, scale_dtype="fp16")[:3], n, k, bits=bits)
        del W
        x = torch.randn(B, k, device="cuda").half()
        for _ in range(4):
            qmm(pk, x)
    else:
        shapes = {r: (n, k) for r, n, k in S.matrices()}
        n, k = {"qkv": shapes["qkv"], "wo": shapes["wo"], "ffn": shapes["gate"], "down": shapes["down"],
                "head": (S.VOCAB, S.D_MODEL)}[args.kernel_case]
        W = torch.randn(n, k, device="cuda") * 0.02
        if args.kernel_case == "ffn":
            g = Q.quantize(W, bits=bits, scale_dtype="fp16")[:3]
            u = Q.quantize(torch.randn(n, k, device="cuda") * 0.02, bits=bits, scale_dtype="fp16")[:3]
            pk = Q.Pack.gateup(g, u, n, k, bits=bits)
            epi = "swiglu"
        else:
            pk = Q.Pack(*Q.quantize(W, bits=bits, scale_dtype="fp16")[:3], n, k, bits=bits)
            epi = "f32"
        del W
        x = torch.randn(args.case_batch or batch, k, device="cuda").half()
        for _ in range(4):
            Q.qmv(pk, x, epi=epi)
    torch.cuda.synchronize()
    if rank == 0:
        print(json.dumps(dict(kernel_case=args.kernel_case, config=args.config, batch=args.case_batch or batch,
                              launches=4)), flush=True)


def tp_block(args, rank, world, local, dist):
    """BASELINE config 5 in the same process as the replica line: the InternLM2.5-7B shape (4-bit), 64 sequences at
    8,192-token histories, tensor parallel over all `world` ranks (strong scaling: the same work at every N).
    Device time of K steps (max over ranks), the per-GPU step roofline, the per-layer time of the o_proj and down
    groups (GEMM + all-reduce, from a per-kind CUDA-event profile) and the all-reduce path that ran."""
    import ctypes as C

    import torch
    from agxforge.inference import assemble
    from agxforge_b200 import _native as N
    model, bits, batch, hist = CONFIGS["internlm7b-q4-8192-b64-tp"]
    K = min(args.steps, args.tp_steps)
    W = 3
    cap = hist + W + K + 2 * args.profile_steps + 4
    m = assemble.build(dict(model=model, bits=bits, batch=batch, cap=cap, seed=4, tp=world,
                            tp_rank=rank if world > 1 else 0), device=local)
    S = m.shape
    rng = np.random.default_rng(8192)
    for b in range(batch):
        m.start(b, [int(rng.integers(0, S.VOCAB))])
        m.fill_history(b, hist - W, seed=8192 + b)
    m.decode(W, want_tokens=False)
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    _, _, t = m.decode(K, want_tokens=False)
    gpu_ms = t["gpu_ms"]
    if dist is not None:
        tt = torch.tensor([gpu_ms], device="cuda")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        gpu_ms = float(tt.item())
    kind_ms = (C.c_float * 6)()
    kind_n = (C.c_int32 * 6)()
    N.check(N.lib().agxc_model_profile(m.handle, args.profile_steps, kind_ms, kind_n), "profile")
    prof = [kind_ms[i] for i in range(6)]
    if dist is not None:
        tt = torch.tensor(prof, device="cuda")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        prof = [float(x) for x in tt.tolist()]
    per_layer_us = {KIND_NAMES[i]: round(1e3 * prof[i] / max(1, kind_n[i]), 2) for i in range(6)}
    kv = batch * S.LAYERS * (S.KV_HEADS // world) * S.HEAD_DIM * 2 * 2 * (hist + (K - 1) / 2.0 + 1)
    step_bytes_gpu = m.weight_bytes + kv
    step_s = gpu_ms / 1e3 / K
    plans = m.plan_info()["tp"]
    out = dict(config="internlm7b-q4-8192-b64-tp", model=model, batch=batch, history=hist, tp=world, steps=K,
               value=round(batch * K / (gpu_ms / 1e3), 1), unit="tok/s", ms_per_step=round(gpu_ms / K, 3),
               scaling="strong", per_gpu_step_roofline=dict(achieved=round(step_bytes_gpu / step_s / 1e9, 1),
                                                          bytes_per_step=int(step_bytes_gpu)),
               per_layer_us=per_layer_us,
               o_proj_group_us=per_layer_us["wo"], down_group_us=per_layer_us["down"],
               allreduce=("none (one device)" if world == 1 else
                          ("fused peer stores, two-shot" if plans["two_shot"] else "fused peer stores, one-shot")
                          if plans["fused"] else "NCCL all-reduce"))
    m.close()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="internlm-q4-1792", choices=sorted(CONFIGS) + sorted(ENCODER_CONFIGS))
    ap.add_argument("--cpu-tokens", type=int, default=2, help="whole tokens the cpu_baseline leg times")
    ap.add_argument("--ref-steps", type=int, default=1)
    ap.add_argument("--profile-steps", type=int, default=4)
    ap.add_argument("--tp-steps", type=int, default=16, help="timed steps of the tensor-parallel block")
    ap.add_argument("--no-tp", action="store_true", help="skip the tensor-parallel block (config 5)")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--tp-allreduce", default="fused", choices=["fused", "nccl"],
                    help="tensor-parallel configs: GEMM + peer-memory all-reduce (fused) or NCCL all-reduce")
    ap.add_argument("--kernel-case", choices=KIND_NAMES, default=None)
    ap.add_argument("--trace-step", action="store_true")
    ap.add_argument("--case-batch", type=int, default=0,
                    help="activation rows of --kernel-case (default: the config's batch; >= 32 = tensor-core qmm)")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be at least 3")

    rank, world, local, dist = dist_setup(args.gpus)
    if args.config in ENCODER_CONFIGS:
        if args.impl == "reference":
            if rank == 0:
                run_encoder_reference(args)
        else:
            run_encoder(args, rank, world, local, dist)
        if dist is not None:
            dist.destroy_process_group()
        return
    if args.impl == "reference":
        if rank == 0:
            run_reference(args, rank, world)
        if dist is not None:
            dist.destroy_process_group()
        return

    import torch
    from agxforge.inference import assemble
    if args.kernel_case:
        kernel_case(args, rank)
        if dist is not None:
            dist.destroy_process_group()
        return
    if args.trace_step:
        if rank == 0:
            trace_step(args)
        if dist is not None:
            dist.destroy_process_group()
        return

    model, bits, batch, hist = CONFIGS[args.config]
    K, W = args.steps, args.warmup
    # timed, e2e (sizing + two runs), profiled and the other batch-1 path's steps: no position clamps
    cap = hist + 5 * K + W + args.profile_steps + 8
    tp = world if args.config in TP_CONFIGS else 1
    rseed = 0 if tp > 1 else rank        # tensor parallel ranks hold shards of ONE model and the same sequences
    keep = bool(rank == 0 and world == 1 and not args.no_cpu)
    m = assemble.build(dict(model=model, bits=bits, batch=batch, cap=cap, seed=2 + rseed, tp=tp,
                            tp_rank=rank if tp > 1 else 0), device=local, keep_packs=keep)
    S = m.shape
    if tp > 1 and args.tp_allreduce == "nccl":
        m.set_option("tp_fused", 0)
    rng = np.random.default_rng(1792 + rseed)
    # the history: positions 0 .. hist - W - 1 filled on the device (seeded), a random current token; then W warm-up
    # steps at positions hist - W .. hist - 1; the timed steps are at positions hist .. hist + K - 1
    for b in range(batch):
        m.start(b, [int(rng.integers(0, S.VOCAB))])
        m.fill_history(b, hist - W, seed=1792 + 7 * rseed + b)
    m.decode(W, want_tokens=False)
    torch.cuda.synchronize()

    # ---- timed: K graph replays back to back, CUDA events on the library's stream
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    clk = Clocks(local).start()
    clk.mark_start()
    _, _, t = m.decode(K, want_tokens=False)
    torch.cuda.synchronize()
    clk.mark_end()
    clk.stop()
    gpu_ms = t["gpu_ms"]
    launches = t["launches_per_step"]
    if dist is not None:
        tt = torch.tensor([gpu_ms], device="cuda")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        gpu_ms = float(tt.item())
        dist.barrier()
    replicas = world if tp == 1 else 1
    tok_s = replicas * batch * K / (gpu_ms / 1e3)

    # ---- e2e: the same number of steps through the C-ABI decode call, host input and output every step
    if dist is not None:
        dist.barrier()
    forced = np.full((K, batch), 0xFFFFFFFF, np.uint64)     # the step's input: "no forced token" (4 B per seq)
    m.decode(K, forced=forced, want_tokens=True, sync_each=2)  # untimed: sizes the call's pinned host buffers
    if dist is not None:
        dist.barrier()
    t0 = time.perf_counter()
    _, _, te = m.decode(K, forced=forced, want_tokens=True, sync_each=2)
    e2e_s = time.perf_counter() - t0
    if dist is not None:
        dist.barrier()
    t0 = time.perf_counter()
    m.decode(K, forced=forced, want_tokens=True, sync_each=1)
    lock_s = time.perf_counter() - t0
    if dist is not None:
        tt = torch.tensor([e2e_s, lock_s], device="cuda")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e2e_s, lock_s = float(tt[0].item()), float(tt[1].item())
    e2e_tok_s = replicas * batch * K / e2e_s
    lock_tok_s = replicas * batch * K / lock_s

    # ---- per-kernel profile (CUDA events around every launch, no overlap) -> the dominant kernel's roofline
    import ctypes as C
    from agxforge_b200 import _native as N
    kind_ms = (C.c_float * 6)()
    kind_n = (C.c_int32 * 6)()
    N.check(N.lib().agxc_model_profile(m.handle, args.profile_steps, kind_ms, kind_n), "profile")
    pos_mid = hist + 4 * K + args.profile_steps // 2  # the profiled steps follow the timed and the e2e steps
    # this rank's shapes (the whole model at tp 1)
    hl, kvl, fl, hd, d = S.HEADS // tp, S.KV_HEADS // tp, S.FFN // tp, S.HEAD_DIM, S.D_MODEL
    kvrow = 2 * kvl * hd * 2                                       # K+V bytes per position per layer

    def pack_bytes(n, k):
        return n * k * bits // 8 + (n * k // 64) * 4
    kind_bytes = {
        "qkv": pack_bytes((hl + 2 * kvl) * hd, d),
        "attn": batch * kvrow * (pos_mid + 1),
        "wo": pack_bytes(d, hl * hd),
        "ffn": 2 * pack_bytes(fl, d),
        "down": pack_bytes(d, fl),
        "head": pack_bytes(m.vocab_count, d),
    }
    total_ms = sum(kind_ms[i] for i in range(6))
    dom = max(range(6), key=lambda i: kind_ms[i])
    dname = KIND_NAMES[dom]
    per_launch_ms = kind_ms[dom] / max(1, kind_n[dom])
    peak, peak_kind = peaks()
    achieved = kind_bytes[dname] / (per_launch_ms / 1e3) / 1e9
    kinds = {KIND_NAMES[i]: dict(launches=int(kind_n[i]), ms=round(kind_ms[i], 4),
                                 share=round(kind_ms[i] / total_ms, 4) if total_ms else None,
                                 us_per_launch=round(1e3 * kind_ms[i] / max(1, kind_n[i]), 3),
                                 gbs=round(kind_bytes[KIND_NAMES[i]] / (kind_ms[i] / max(1, kind_n[i]) / 1e3) / 1e9, 1)
                                 if kind_ms[i] > 0 else None) for i in range(6)}
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "traffic.md")
    if os.path.exists(tpath):
        for ln in open(tpath):
            if ln.startswith("traffic %s %s " % (args.config, dname)):
                try:
                    traffic = int(ln.split()[3])
                except (IndexError, ValueError):
                    traffic = None

    # the other batch-1 path on the same model (the fused persistent step when the graph is the default, or the
    # reverse): W warm-up and K timed steps after the profiled ones, device time; reported beside, not in, the value
    other = None
    if batch == 1 and tp == 1 and m.plan_info()["fused"]["fits"]:
        was = m.fused
        m.set_option("fused", 0 if was else 1)
        m.decode(W, want_tokens=False)
        _, _, to = m.decode(K, want_tokens=False)
        m.set_option("fused", 1 if was else 0)
        other = dict(path="graph (one kernel per projection)" if was else "fused persistent step",
                     tok_s=round(K / (to["gpu_ms"] / 1e3), 2), ms_per_step=round(to["gpu_ms"] / K, 4),
                     launches_per_step=to["launches_per_step"],
                     positions=[hist + 4 * K + args.profile_steps + W, hist + 5 * K + args.profile_steps + W - 1])

    # whole-step algorithmic bytes: every pack once + every sequence's KV over the timed positions (mean)
    w_bytes = m.weight_bytes
    kv_bytes = batch * S.LAYERS * kvrow * (hist + (K - 1) / 2.0 + 1)
    step_bytes = w_bytes + kv_bytes
    step_s = gpu_ms / 1e3 / K
    step_gbs = step_bytes / step_s / 1e9

    # the prefill section on the same model: the history as a prompt of `hist` tokens (positions 0 .. hist-2 through
    # the tensor-core GEMMs and the causal prefill attention), one warm-up then one timed run (device time)
    prefill = None
    if tp == 1 and S.QKV % 128 == 0 and S.D_MODEL % 128 == 0:
        prompt = rng.integers(0, S.VOCAB, hist).tolist()
        m.prefill(0, prompt)
        pt = m.prefill(0, prompt)
        prefill = dict(tokens=hist - 1, gpu_ms=round(pt["gpu_ms"], 3),
                       tok_s=round((hist - 1) / (pt["gpu_ms"] / 1e3), 1), launches=pt["launches"])

    # the dominant kernel: the fused step when it runs (the step's only launch; its device time is the timed
    # replays'), else the per-kernel path's largest share
    fused = batch == 1 and tp == 1 and m.fused
    if fused:
        us = gpu_ms / K * 1e3
        ftraffic = None
        for ln in (open(tpath) if os.path.exists(tpath) else []):
            if ln.startswith("traffic %s fused " % args.config):
                try:
                    ftraffic = int(ln.split()[3])
                except (IndexError, ValueError):
                    ftraffic = None
        roofline = dict(bound="hbm", kernel="fused_step", achieved=round(step_gbs, 1), peak=peak, unit="GB/s",
                        frac=round(step_gbs / peak, 4), traffic=ftraffic, peak_source=peak_kind,
                        bytes_per_launch=int(step_bytes), us_per_launch=round(us, 3),
                        timing="CUDA events on the library's stream around the K timed steps (one launch a step)")
    else:
        roofline = dict(bound="hbm", kernel=dname, achieved=round(achieved, 1), peak=peak, unit="GB/s",
                        frac=round(achieved / peak, 4), traffic=traffic, peak_source=peak_kind,
                        bytes_per_launch=kind_bytes[dname], us_per_launch=round(per_launch_ms * 1e3, 3))

    cpu = None
    if keep:
        per_token, cores = cpu_baseline_sample(m, args.cpu_tokens, hist)
        cpu = dict(value=round(1.0 / per_token, 5), unit="tok/s", cores=cores,
                   cpu=cpu_model(), kind="port",
                   sample="%d whole tokens (all %d layers, head, argmax) of one sequence at position %d over a seeded "
                          "history, this run's packs copied to the host (%.2f s a token)%s" % (
                              args.cpu_tokens, S.LAYERS, hist, per_token,
                              "; the CPU step is per sequence, so a batch of %d takes %d such tokens" % (batch, batch)
                              if batch > 1 else ""))

    if rank == 0:
        line = dict(
            metric=METRIC, value=round(tok_s, 2), unit="tok/s", n_gpus=world, steps=K, warmup=W,
            ms_per_step=round(gpu_ms / K, 4), higher_is_better=True, scaling="strong" if tp > 1 else "weak",
            vs_baseline=None, dtype="u4" if
            bits == 4 else "u8", data="synthetic (seeded random-init weights and uniform-random token ids)",
            config=workload_config(args, world, model, bits, batch, hist, tp),
            e2e=dict(value=round(e2e_tok_s, 2), unit="tok/s", h2d_bytes_per_step=4 * batch,
                     d2h_bytes_per_step=4 * batch, loop="one step queued ahead (sync_each 2)",
                     lockstep=round(lock_tok_s, 2)),
            roofline=roofline,
            step_roofline=dict(bound="hbm", achieved=round(step_gbs, 1), peak=peak, unit="GB/s",
                               frac=round(step_gbs / peak, 4), bytes_per_token=int(step_bytes / batch),
                               weight_bytes=w_bytes, peak_source=peak_kind),
            kernels=kinds if not fused else None,
            graph_path_kernels=kinds if fused else None,
            other_path=other,
            prefill=prefill,
            plans=m.plan_info(),
            cpu_baseline=cpu,
            clocks=clk.summary(),
            gpu_launches=int(launches * K),
        )
    m.close()
    torch.cuda.synchronize()
    tp_failed = False
    if args.config == "internlm-q4-1792" and not args.no_tp:
        try:
            tpb = tp_block(args, rank, world, local, dist)
        except Exception as e:  # the replica line stands; the tensor-parallel block reports what went wrong
            tpb = dict(error="%s: %s" % (type(e).__name__, str(e)[:300]))
            tp_failed = True
        if rank == 0:
            line["tp"] = tpb
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist is not None:
        try:
            dist.barrier()
            dist.destroy_process_group()
        except Exception:
            if not tp_failed:  # a communicator broken by the failed block may not close cleanly
                raise


if __name__ == "__main__":
    main()
