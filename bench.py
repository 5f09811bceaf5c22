#!/usr/bin/env python
"""Benchmark: Q4_K GEMV achieved HBM GB/s on B200.

Workload: y = W . x with W a Q4_K matrix of N=4096 rows x K=4096 columns
(65,536 blocks, 9,437,184 bytes), x and y fp32, M=1 -- the single Q4_K GEMV
of the headline metric, seeded as its definition says (d = fp16(|N(0,1)|*2e-3),
dmin = fp16(|N(0,1)|*1e-3), scales/mins uniform 0..63, nibbles uniform).
A step is one GEMV over each of COPIES distinct weight matrices (64 x 9.4 MB
= 604 MB, more than 4x the 126 MB L2, so every step streams from HBM).  The
COPIES launches of a step are one CUDA graph; the timed region replays it.

--workload gemm measures the prefill dequant-GEMM instead (one line, not the
headline): Y[M x N] = X[M x K] . W^T for the Llama-3-8B FFN up-projection
shape N=14336, K=4096 (default Q4_K, M=512), rotating over weight copies that
exceed 4x L2, through swq_gemm on the tensor cores.

Arms:
  --impl swq (default): libswq on each GPU.  Under torchrun every rank runs
      its own stream of GEMVs on its own weights (weak scaling, no data-path
      collective); the time is the max over ranks.
  --impl reference: the reference's own CPU code (Compute::matmul_transposed_q,
      compiled from source into oracle/_ref; the oracle port if that is
      absent) on all host cores, one Q4_K 4096x4096 GEMV per step; and, in
      "decode", the reference's Model::forward tok/s on a Llama-3-8B-shaped
      Q4_K_M GGUF file written for the run (src/model.h compiled from source).

One JSON line on rank 0.
"""
from __future__ import annotations

import argparse
import csv
import io
import json
import os
import shutil
import statistics
import subprocess
import sys
import time


from pathlib import Path  # noqa: E402

REPO = Path(__file__).resolve().parent
for _p in (str(REPO), str(REPO / "swllm.cpp_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "Q4_K GEMV achieved HBM GB/s (% peak); decode tok/s at 1/2/4/8 B200"
DECODE_DEADLINE_S = 540  # decode and MoE measurements of the default run (about 90 s on one GPU)
N_ROWS, K_COLS, M_ROWS = 4096, 4096, 1
COPIES = 64
REPLAYS = 128       # graph replays per step: a step is REPLAYS x COPIES GEMVs
GEMV_STREAMS = 4    # streams the COPIES independent GEMVs of a graph alternate over
GEMV_CTAS_PER_SM = 3  # SWQ_OPT_GEMV_CTAS_PER_SM for them: three GEMVs (CTAs of 8 warps) on each SM at once
REF_STEP_GEMVS = 64  # GEMVs per step of the reference arm
Q4_K = 12
BLOCK_BYTES = 144
W_BYTES = N_ROWS * (K_COLS // 256) * BLOCK_BYTES              # 9,437,184
ALG_BYTES = W_BYTES + 4 * K_COLS * M_ROWS + 4 * N_ROWS * M_ROWS  # 9,469,952 per GEMV
WORKLOAD = (f"Q4_K GEMV N={N_ROWS} K={K_COLS} M={M_ROWS}, {COPIES} rotating weight copies "
            f"({COPIES * W_BYTES / 1e6:.0f} MB)")
# dram__bytes_read.sum + dram__bytes_write.sum of one gemv_kq_kernel<Q4_K, 8>
# launch of this workload (the launch shape of the timed graph): the mean of
# three launches of one ncu capture (profiles/gemv_kq_q4k_4096x4096.md:
# 9,492,992 / 9,491,968 / 9,496,576 read, 0 written).
NCU_TRAFFIC_PER_LAUNCH = 9493845


_T0 = time.time()


def log(*a):
    print(f"[{time.time() - _T0:7.1f}s]", *a, file=sys.stderr, flush=True)


# The result is the one JSON line on stdout.  Libraries write to stdout too
# (NCCL's "NCCL version" banner at its default log level), so main() moves
# file descriptor 1 onto stderr and keeps the original stdout for emit().
_RESULT_OUT = None


def _claim_stdout() -> None:
    global _RESULT_OUT
    if _RESULT_OUT is None:
        sys.stdout.flush()
        _RESULT_OUT = os.fdopen(os.dup(1), "w")
        os.dup2(2, 1)


def emit(line: dict) -> None:
    """Print the result line on the original stdout."""
    out = _RESULT_OUT if _RESULT_OUT is not None else sys.stdout
    print(json.dumps(line), file=out, flush=True)


def _gemv_form(fmt: str, M: int) -> str:
    """The GEMV kernel the library picks for `fmt` at M rows (default options)."""
    if M == 1 and fmt in ("Q4_K", "Q6_K"):
        return f"swq::kq::gemv_kq_kernel<{fmt}> (30-bit fixed-point x, exact integer sub-block sums)"
    if fmt in ("Q4_K", "Q6_K") and 2 <= M <= 16:
        return (f"swq::kqm::gemv_kqm_kernel<{fmt}> (x as fp16 pairs per super-block, exact products, "
                f"fp32 sums)")
    return f"swq::gemv_kernel<{fmt},M> (fp32 x, fp32 FMA)"


def _batched_path(fmt: str, M: int) -> bool:
    """True where the batched K-quant GEMV serves M rows (default options)."""
    return fmt in ("Q4_K", "Q6_K") and 2 <= M <= 16


def load_peaks() -> tuple[float, str]:
    p = REPO / "MEASURED_PEAKS.json"
    try:
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def load_tensor_peak() -> tuple[float, str]:
    """Dense bf16 TFLOP/s of this pool's B200s: the burst figure (a kernel
    timed in a loop of well under a second is not power-capped for long)."""
    p = REPO / "MEASURED_PEAKS.json"
    try:
        d = json.loads(p.read_text())
        return float(d["bf16_tflops"]), "measured (burst)"
    except Exception:
        return 1590.0, "fallback"


# ---------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.gpu_id = gpu_id
        self.proc = None
        self.err = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu_id}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True)
        except Exception as e:  # pragma: no cover
            self.err = str(e)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out, _ = self.proc.communicate()

    def summary(self) -> dict:
        if self.proc is None:
            return {"unavailable": self.err or "nvidia-smi not started"}
        rows = [r for r in csv.reader(io.StringIO(self.out or "")) if len(r) >= 9]
        if not rows:
            return {"unavailable": "no nvidia-smi samples during the timed region"}
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        smax = [float(r[2]) for r in rows if r[2].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].strip() == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "reasons": reasons, "samples": len(rows)}


class _NoClock:
    def __enter__(self):
        return self

    def __exit__(self, *exc):
        pass

    def summary(self) -> dict:
        return {}


# ---------------------------------------------------------------- CPU arm
def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for ln in f:
                if ln.startswith("model name"):
                    return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_gemv_timing(seconds: float, min_steps: int = 1, copies: int = 16, threads: int = 0, warmup: int = 1,
                    per_step: int = 1) -> dict:
    """The reference CPU routine on all host cores (or `threads`): steps of
    `per_step` Q4_K 4096x4096 GEMVs rotating over `copies` weight matrices
    (151 MB, beyond the LLC), after `warmup` untimed GEMVs; at least
    `min_steps` steps and at least `seconds` of timed work."""
    import numpy as np

    import oracle
    from swq import synth

    cores = threads or oracle.host_cores()
    if oracle.ref_available():
        kind = "reference"
        oracle.ref_set_threads(cores)
        fn = lambda w, x: oracle.ref_gemv(Q4_K, w, x, N_ROWS, K_COLS)  # noqa: E731
    else:
        kind = "port"
        oracle.set_threads(cores)
        fn = lambda w, x: oracle.gemv(Q4_K, w, x, N_ROWS, K_COLS)  # noqa: E731
    ws = [synth.random_blocks(Q4_K, N_ROWS, K_COLS, seed=1000 + i) for i in range(copies)]
    x = synth.random_activations(1, K_COLS, seed=7)[0]
    for i in range(max(1, warmup)):
        fn(ws[i % copies], x)
    n = steps = 0
    t0 = time.perf_counter()
    while True:
        for _ in range(per_step):
            fn(ws[n % copies], x)
            n += 1
        steps += 1
        el = time.perf_counter() - t0
        if el >= seconds and steps >= min_steps:
            break
    gbs = n * ALG_BYTES / el / 1e9
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": kind,
            "sample": f"{n} Q4_K GEMVs N={N_ROWS} K={K_COLS} M=1 over {copies} weight copies "
                      f"({steps} steps of {per_step}), {el:.1f} s, {cores} OpenMP threads, after "
                      f"{max(1, warmup)} warm-up GEMVs", "seconds": round(el, 2), "steps": steps, "gemvs": n}


def write_llama_gguf(path, cfg, seed: int = 0) -> int:
    """A GGUF file of `cfg`'s dense Llama shape with synthetic weights in its
    type mix (the metric's block distributions, a Q4_K embedding table as in
    a Q4_K_M file, norms 1 + N(0, 0.01)), written one tensor at a time.
    Returns the file's size."""
    import numpy as np

    from swq import gguf as G
    from swq import synth

    stems = {"wq": "attn_q", "wk": "attn_k", "wv": "attn_v", "wo": "attn_output", "w_gate": "ffn_gate",
             "w_up": "ffn_up", "w_down": "ffn_down"}
    rng = np.random.default_rng(seed)
    meta = {"general.architecture": "llama", "general.name": "synthetic",
            "llama.context_length": cfg.max_seq, "llama.embedding_length": cfg.dim,
            "llama.block_count": cfg.n_layers, "llama.feed_forward_length": cfg.ffn,
            "llama.attention.head_count": cfg.n_heads, "llama.attention.head_count_kv": cfg.n_kv_heads,
            "llama.rope.freq_base": G.GGUFValue(G.FLOAT32, cfg.theta),
            "llama.attention.layer_norm_rms_epsilon": G.GGUFValue(G.FLOAT32, cfg.eps),
            "llama.vocab_size": cfg.vocab, "tokenizer.ggml.model": "llama",
            "tokenizer.ggml.tokens": [f"<{i}>" for i in range(cfg.vocab)]}
    mats = lambda t, N, K, sd: (lambda: synth.fast_random_blocks(t, N, K, seed=sd))  # noqa: E731
    norm = lambda: (1 + 0.01 * rng.standard_normal(cfg.dim)).astype(np.float32)  # noqa: E731
    tensors = [("token_embd.weight", G.Q4_K, (cfg.dim, cfg.vocab), mats(G.Q4_K, cfg.vocab, cfg.dim, seed + 1)),
               ("output_norm.weight", G.F32, (cfg.dim,), norm()),
               ("output.weight", cfg.types["output"], (cfg.dim, cfg.vocab),
                mats(cfg.types["output"], cfg.vocab, cfg.dim, seed + 2))]
    for li in range(cfg.n_layers):
        lt = cfg.layer_type_map(li)
        tensors += [(f"blk.{li}.attn_norm.weight", G.F32, (cfg.dim,), norm()),
                    (f"blk.{li}.ffn_norm.weight", G.F32, (cfg.dim,), norm())]
        for j, (key, (N, K)) in enumerate(cfg.shapes().items()):
            tensors.append((f"blk.{li}.{stems[key]}.weight", lt[key], (K, N),
                            mats(lt[key], N, K, seed + 100 + 10 * li + j)))
    G.write_gguf(path, meta, tensors)
    return os.path.getsize(path)


def _mem_available() -> int:
    try:
        with open("/proc/meminfo") as f:
            for ln in f:
                if ln.startswith("MemAvailable:"):
                    return int(ln.split()[1]) * 1024
    except OSError:
        pass
    return 0


def ref_decode_timing(cfg, seconds: float = 20.0, max_tokens: int = 8, workdir: str | None = None) -> dict:
    """The reference's own decode on the host cores: Model::load of a GGUF file
    of `cfg`'s shape (written here, deleted once loaded -- the reference keeps
    the whole file in memory), then Model::forward calls at positions 0, 1,
    2, ... on seeded token ids (teacher-forced), timed with the wall clock
    after one warm-up call.  The context stays short, so the reference reads less
    KV per token than after a real prefill (its number is, if anything, high)."""
    import tempfile

    import numpy as np

    import oracle
    from oracle.ref_model import RefModel, model_ref_available

    if not model_ref_available():
        return {"unavailable": "the reference's model library was not built (oracle/_ref)"}
    est = cfg.weight_bytes_per_token() + cfg.vocab * cfg.dim * 144 // 256
    if workdir is None:  # memory-backed when it has room: the reference freads the whole file
        roomy = [d for d in ("/dev/shm", tempfile.gettempdir())
                 if os.path.isdir(d) and os.access(d, os.W_OK) and shutil.disk_usage(d).free >= est + (2 << 30)]
        workdir = roomy[0] if roomy else tempfile.gettempdir()
    free = shutil.disk_usage(workdir).free
    if free < est + (2 << 30):
        return {"unavailable": f"{free / 1e9:.1f} GB free in {workdir}, the model file needs {est / 1e9:.1f} GB"}
    need_ram = est + cfg.vocab * cfg.dim * 4 + (4 << 30)  # the file in memory + the fp32 embedding table
    if workdir.startswith("/dev/shm"):  # the file itself sits in memory until it is loaded and deleted
        need_ram += est
    if 0 < _mem_available() < need_ram:
        return {"unavailable": f"{_mem_available() / 1e9:.1f} GB of host memory available, "
                               f"{need_ram / 1e9:.1f} GB needed"}
    cores = oracle.host_cores()
    t0 = time.perf_counter()
    with tempfile.TemporaryDirectory(dir=workdir) as d:
        path = os.path.join(d, "model.gguf")
        size = write_llama_gguf(path, cfg)
        t_write = time.perf_counter() - t0
        m = RefModel(path)
        os.unlink(path)
    t_load = time.perf_counter() - t0 - t_write
    toks = np.random.default_rng(3).integers(0, cfg.vocab, size=max_tokens + 1).tolist()
    finite = bool(np.isfinite(m.forward(toks[0], 0)).all())  # warm-up
    n, t1 = 0, time.perf_counter()
    while n < max_tokens:
        finite &= bool(np.isfinite(m.forward(toks[n + 1], n + 1)).all())
        n += 1
        if time.perf_counter() - t1 >= seconds:
            break
    el = time.perf_counter() - t1
    m.close()
    per_tok = el / n
    return {"tok_s": round(1.0 / per_tok, 3), "ms_per_step": round(1e3 * per_tok, 2),
            "weight_GBps": round(cfg.weight_bytes_per_token() / per_tok / 1e9, 2), "finite_logits": finite,
            "cores": cores, "kind": "reference",
            "sample": f"{n} Model::forward calls at positions 1..{n} after one warm-up call, {el:.1f} s, "
                      f"{cores} OpenMP threads; model file {size / 1e9:.2f} GB written to {workdir} in "
                      f"{t_write:.1f} s, loaded in {t_load:.1f} s (not timed)"}


def run_reference(args, rank: int) -> None:
    if rank != 0:
        return
    # steps of 64 GEMVs (one graph's worth of the GPU arm), --steps of them
    # and at least 10 s of timed CPU work, after --warmup warm-up GEMVs
    r = cpu_gemv_timing(seconds=10.0, min_steps=max(1, args.steps), warmup=args.warmup, per_step=REF_STEP_GEMVS)
    one = cpu_gemv_timing(seconds=5.0, copies=4, threads=1, warmup=1, per_step=1)
    import oracle
    (oracle.ref_set_threads if oracle.ref_available() else oracle.set_threads)(oracle.host_cores())
    line = {"impl": "reference", "metric": METRIC, "value": r["value"], "unit": "GB/s",
            "n_gpus": args.gpus, "steps": r["steps"], "warmup": args.warmup, "steps_requested": args.steps,
            "ms_per_step": round(1e3 * r["seconds"] / r["steps"], 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"Q4_K GEMV N={N_ROWS} K={K_COLS} M=1 (reference CPU path)",
                       "format": "Q4_K", "N": N_ROWS, "K": K_COLS, "M": 1},
            "cpu_baseline": {"value": r["value"], "unit": "GB/s", "cores": r["cores"], "kind": r["kind"],
                             "sample": r["sample"], "cpu_model": cpu_model(),
                             "single_thread": {"value": one["value"], "unit": "GB/s", "sample": one["sample"]}},
            "e2e": {"value": r["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    if args.decode:
        from swq.model import LlamaConfig
        cfg = LlamaConfig(max_seq=1024)
        log("reference decode: writing and loading the Llama-3-8B-shaped GGUF")
        try:
            dec = ref_decode_timing(cfg, seconds=20.0, max_tokens=max(2, min(args.steps, 16)))
        except Exception as e:  # the GEMV line stands without it
            dec = {"unavailable": f"{type(e).__name__}: {e}"}
        line["decode"] = {
            "model": "Llama-3-8B shape, Q4_K_M mix (Q6_K attn_v/ffn_down/output, Q4_K else), synthetic weights",
            "weight_bytes_per_token": cfg.weight_bytes_per_token(),
            "note": "the reference's Model::forward decodes one sequence per call (src/main.cpp), so a batch "
                    "of B sequences takes B calls: its tok/s is the same at every batch size",
            "batches": {"1": dec}}
    emit(line)


# ---------------------------------------------------------------- GPU arm
def run_swq(args, rank: int, world: int) -> None:
    import numpy as np
    import torch

    import swq
    from swq import synth

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=dev)

    log(f"gemv: rank {rank}/{world} building {COPIES} weight copies")
    # Weights: COPIES distinct seeded matrices per rank, resident in HBM.
    host_ws = [synth.random_blocks(Q4_K, N_ROWS, K_COLS, seed=10_000 * rank + i) for i in range(COPIES)]
    d_ws = [torch.from_numpy(w.reshape(-1)).to(dev) for w in host_ws]
    x_host = synth.random_activations(1, K_COLS, seed=5 + rank)
    d_x = torch.from_numpy(x_host).to(dev)
    d_ys = [torch.empty(N_ROWS, dtype=torch.float32, device=dev) for _ in range(COPIES)]

    torch.cuda.synchronize()

    def capture(nstreams: int, ctas: int = 0):
        """One CUDA graph of the COPIES GEMVs, launch i on stream i % nstreams:
        the graph holds no edge between GEMVs of different streams (they are
        independent: same x, their own W and y), so their kernels may run at
        the same time; on one stream each waits for its predecessor
        (programmatic dependent launch: its weights stream in early, x is
        read after the predecessor completes)."""
        streams = [torch.cuda.Stream(device=dev) for _ in range(nstreams)]
        main = streams[0]

        def issue():
            fork = torch.cuda.Event()
            fork.record(main)
            for st in streams[1:]:
                st.wait_event(fork)
            for i in range(COPIES):
                st = streams[i % nstreams]
                swq.gemv(Q4_K, d_ws[i], d_x, d_ys[i], N_ROWS, K_COLS, stream=st)
            for st in streams[1:]:
                join = torch.cuda.Event()
                join.record(st)
                main.wait_event(join)

        old = swq.get_option(swq.OPT_GEMV_CTAS_PER_SM)
        swq.set_option(swq.OPT_GEMV_CTAS_PER_SM, ctas)  # read at launch: the graph keeps this launch shape
        with torch.cuda.stream(main):
            issue()  # eager warm-up: attributes set, kernels loaded
        swq.check(main)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=main):
            issue()
        swq.set_option(swq.OPT_GEMV_CTAS_PER_SM, old)
        return g, main

    def time_steps(g, st, steps: int, warmup: int, clocks: bool):
        with torch.cuda.stream(st):
            for _ in range(warmup * REPLAYS):
                g.replay()
        st.synchronize()
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(gpu_uuid) if clocks else _NoClock() as clk:
            with torch.cuda.stream(st):
                ev0.record(st)
                for _ in range(steps * REPLAYS):
                    g.replay()
                ev1.record(st)
            ev1.synchronize()
        torch.cuda.synchronize()
        ms = ev0.elapsed_time(ev1)
        swq.check(st)
        if dist:
            t = torch.tensor([ms], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
            dist.barrier()
        return ms, clk.summary()

    peak, peak_kind = load_peaks()
    gpu_uuid = str(torch.cuda.get_device_properties(dev).uuid)
    gpu_uuid = gpu_uuid if gpu_uuid.startswith("GPU-") else f"GPU-{gpu_uuid}"
    graph, stream = capture(GEMV_STREAMS, GEMV_CTAS_PER_SM)
    graph1, stream1 = capture(1)
    log(f"gemv: timing {args.steps} steps of {REPLAYS} x {COPIES} GEMVs on {GEMV_STREAMS} streams")
    ms, clocks = time_steps(graph, stream, args.steps, max(3, args.warmup), clocks=True)
    chain_steps = max(1, min(args.steps, 10))
    ms1, _ = time_steps(graph1, stream1, chain_steps, 3, clocks=False)
    launches = args.steps * REPLAYS * COPIES
    total_bytes = launches * ALG_BYTES * world
    value = total_bytes / (ms * 1e-3) / 1e9
    per_launch_s = ms * 1e-3 / launches
    achieved = ALG_BYTES / per_launch_s / 1e9
    chain_launch_s = ms1 * 1e-3 / (chain_steps * REPLAYS * COPIES)

    # The host-buffer path below must reproduce the device result of the last copy.
    y_last = d_ys[-1].cpu().numpy()

    # End to end through the host-buffer API (the reference's calling
    # convention): host x in, host y out, weights resident after first use.
    # The timed calls go straight to the C ABI, as the reference's C++ call
    # site would make them: raw host pointers held by the caller, one call per
    # GEMV (the Python mirror's per-call argument checks and pointer lookups,
    # about 3 us of a 36 us call on a B200 host, are not part of the drop-in).
    # The warm-up runs through the mirror on the same arrays, so the weights
    # are resident under the same host addresses.
    from swq.lib import _raise, lib as swq_lib
    e2e_steps = max(1, min(args.steps, 200))
    comp = swq.Compute(device=local)
    out = np.zeros(N_ROWS, np.float32)
    x0 = x_host[0]
    qws = [swq.QuantWeight(w, Q4_K) for w in host_ws]
    if not (x0.flags.c_contiguous and all(q.data.flags.c_contiguous and q.data.dtype == np.uint8 for q in qws)):
        raise RuntimeError("e2e: host arrays must be C-contiguous (the mirror would copy them)")
    for i in range(COPIES):  # upload once (warm-up)
        comp.matmul_transposed_q(out, x0, qws[i], N_ROWS, K_COLS)
    fn = swq_lib().swq_ctx_matmul_transposed_q
    ctx, p_out, p_x = comp._ctx, out.ctypes.data, x0.ctypes.data
    p_ws = [q.data.ctypes.data for q in qws]
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        for i in range(COPIES):
            rc = fn(ctx, p_out, p_x, p_ws[i], Q4_K, N_ROWS, K_COLS)
            if rc:
                _raise(rc)
    e2e_s = time.perf_counter() - t0
    if dist:
        t = torch.tensor([e2e_s], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e_value = e2e_steps * COPIES * ALG_BYTES * world / e2e_s / 1e9
    comp.close()
    if not np.allclose(out, y_last, rtol=1e-5, atol=1e-4):
        raise RuntimeError("host-buffer path disagrees with the device path")

    line = None
    if rank == 0:
        cpu = None
        if world == 1:
            cpu = cpu_gemv_timing(seconds=10.0)
            cpu = {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")}
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 5),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic",
            "config": {"workload": WORKLOAD, "format": "Q4_K", "N": N_ROWS, "K": K_COLS, "M": M_ROWS,
                       "copies": COPIES, "gemvs_per_step": REPLAYS * COPIES, "bytes_per_gemv": ALG_BYTES,
                       "issue": f"{COPIES} independent GEMVs (same x, own W and y) per graph, alternating over "
                                f"{GEMV_STREAMS} streams, SWQ_OPT_GEMV_CTAS_PER_SM={GEMV_CTAS_PER_SM} (a CTA of 8 "
                                f"consumer warps per SM and GEMV, three GEMVs per SM at once); consecutive GEMVs of "
                                f"one stream are programmatic dependents (weights prefetched, x read after the "
                                f"predecessor completes)",
                       "l2": "inputs larger than L2 (rotating weights)",
                       "arith": "fp32 activations as 30-bit fixed point per 256-element super-block (4 int8 "
                                "limbs); exact integer sub-block products (mma.sync u8 x s8 -> s32) scaled by the "
                                "6-bit scales in int32; one fp32 conversion per super-block, fp32 sums",
                       "parallelism": f"replicas x{world}" if world > 1 else "single GPU"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                         "traffic": NCU_TRAFFIC_PER_LAUNCH,
                         "kernel": "swq::kq::gemv_kq_kernel<Q4_K,8>", "alg_bytes_per_launch": ALG_BYTES,
                         "us_per_launch": round(per_launch_s * 1e6, 3),
                         "chain": {"us_per_launch": round(chain_launch_s * 1e6, 3),
                                   "achieved": round(ALG_BYTES / chain_launch_s / 1e9, 1),
                                   "frac": round(ALG_BYTES / chain_launch_s / 1e9 / peak, 4),
                                   "note": "the same GEMVs on one stream, default launch shape (two CTAs of "
                                           "16 consumer warps per SM): each waits for its predecessor"}},
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s",
                    "h2d_bytes_per_step": COPIES * 4 * K_COLS * M_ROWS,
                    "d2h_bytes_per_step": COPIES * 4 * N_ROWS * M_ROWS,
                    "api": "swq_ctx_matmul_transposed_q (host fp32 x/out, resident weights; called "
                           "through ctypes with the host pointers taken once, as a C++ call site holds them)",
                    "steps": e2e_steps},
            "gpu_launches": launches,
            "clocks": clocks,
            "decode": None,
            "decode_70b": None,
            "moe": None,
            "moe_decode": None,
        }
    del graph, graph1

    # The decode measurements run under a deadline: if one does not finish
    # (a collective that never completes), rank 0 prints the line with what
    # was measured and a note, and every rank leaves.  Every device-side wait
    # of libswq is bounded, so leaving the process releases the GPU.
    import threading

    def _deadline():
        if line is not None:
            line["decode_timeout"] = f"decode measurements did not finish within {DECODE_DEADLINE_S} s"
            emit(line)
        log("decode deadline reached; exiting")
        os._exit(0 if line is not None or rank != 0 else 1)

    timer = threading.Timer(DECODE_DEADLINE_S, _deadline)
    timer.daemon = True
    timer.start()
    if world == 1 and args.sweep:
        log("gemv: done; config-1 format x batch sweep")
        line["sweep"] = run_sweep()
    if args.decode:
        log("gemv: done; decode next")
        decode = run_decode(rank, world, steps=256)
        if line is not None:
            line["decode"] = decode
        decode_tp = run_decode_tp(rank, world)
        if line is not None:
            line["decode_70b"] = decode_tp
    if args.moe:
        log("gemv: done; MoE layer next")
        moe = run_moe(rank, world)
        if line is not None:
            line["moe"] = moe
        log("gemv: MoE decoder next")
        moe_dec = run_decode_moe(rank, world)
        if line is not None:
            line["moe_decode"] = moe_dec
    timer.cancel()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if line is not None:
        emit(line)


# ---------------------------------------------------------------- prefill workload
def run_prefill(rank: int, prompt: int = 512, reps: int = 3, warmup: int = 1, seventy: bool = False) -> dict:
    """Batched prefill of one `prompt`-token sequence of uniform-random token
    ids through a Llama-3-8B-shaped (or, with seventy, Llama-3-70B-shaped)
    Q4_K_M model with synthetic weights on one GPU: LlamaDecoder.prefill, every
    projection one M-row tensor-core GEMM, CUDA-event timed on the decode
    stream (median of `reps` after `warmup`).  TFLOP/s counts the projections
    only: 2 x prompt x the layers' weight elements, plus the LM head for the
    last row (attention excluded)."""
    import numpy as np
    import torch

    from swq.model import LlamaConfig, LlamaDecoder

    cfg = (LlamaConfig.llama3_70b if seventy else LlamaConfig)(max_seq=prompt + 8)
    dec = LlamaDecoder(cfg, rows=1, seed=300 + rank)
    toks = np.random.default_rng(5).integers(0, cfg.vocab, size=(1, prompt)).tolist()
    # layer projections for every prompt row, the LM head for the last row only
    flops = 2.0 * prompt * cfg.n_layers * sum(n * k for n, k in cfg.shapes().values()) + 2.0 * cfg.vocab * cfg.dim
    ms = []
    for i in range(warmup + reps):
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(dec.stream)
        dec.prefill(toks)
        ev1.record(dec.stream)
        ev1.synchronize()
        if i >= warmup:
            ms.append(ev0.elapsed_time(ev1))
    t = statistics.median(ms)
    return {"model": ("Llama-3-70B" if seventy else "Llama-3-8B") + " shape, Q4_K_M mix, synthetic weights",
            "prompt_tokens": prompt, "ms": round(t, 2), "tok_s": round(prompt / (t * 1e-3), 1),
            "projection_TFLOPs": round(flops / (t * 1e-3) / 1e12, 1),
            "finite_logits": bool(torch.isfinite(dec.logits).all().item()), "reps_ms": [round(x, 2) for x in ms]}


# ---------------------------------------------------------------- decode workload
# How the decode measurements build their context: "synthetic" (random K/V in
# the cache, Decoder.fill_kv) or "prefill" (LlamaDecoder.prefill of uniform
# random prompt tokens, timed on its own and reported as prefill_ms).
DECODE_CONTEXT = "prefill"


def _build_context(dec, n: int, seed: int, share_from=None) -> dict:
    """Positions 0..n-1 of every sequence, then the decoder stands at position n.
    share_from: a one-row decoder of the same model that prefilled the prompt;
    every row of `dec` continues from its cache (one prompt shared by the
    batch: its K/V rows copied, no second prefill)."""
    import numpy as np
    import torch
    if share_from is not None:
        src = share_from
        with torch.cuda.stream(dec.stream):
            dec.stream.wait_stream(src.stream)
            dec.kcache[:, :, :n].copy_(src.kcache[:, :1, :n].expand(-1, dec.rows, -1, -1))
            dec.vcache[:, :, :n].copy_(src.vcache[:, :1, :n].expand(-1, dec.rows, -1, -1))
            dec.tokens.fill_(int(src.history[0, 0].item()))
            dec.history[0].fill_(int(src.history[0, 0].item()))
            dec.pos.fill_(n)
            dec.step_no.fill_(1)
        dec.steps_issued = 1
        return {"context": f"the {n}-token prompt prefilled at batch 1, its K/V shared by the {dec.rows} rows"}
    if DECODE_CONTEXT == "prefill":
        toks = np.random.default_rng(seed).integers(0, dec.cfg.vocab, size=(dec.rows, n)).tolist()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(dec.stream)
        dec.prefill(toks)
        ev1.record(dec.stream)
        ev1.synchronize()
        return {"context": f"prefill of {n} uniform random tokens", "prefill_ms": round(ev0.elapsed_time(ev1), 2)}
    dec.reset([(7 * i + 1) % dec.cfg.vocab for i in range(dec.rows)], 0)
    dec.fill_kv(n)
    return {"context": f"synthetic K/V for {n} positions"}

def run_decode(rank: int, world: int, batches=(1, 16), prefill: int = 512, steps: int = 256,
               warmup: int = 5, gguf: str | None = None) -> dict:
    """Greedy decode of a Llama-3-8B-shaped model (32 layers, hidden 4096,
    32/8 heads of 128, FFN 14336, vocab 128256, Q4_K_M mix, synthetic weights
    generated on the device) after a synthetic 512-token context: `steps`
    graph-replayed steps per batch size, CUDA-event timed.  Every rank runs its
    own model (replicas); tok/s is summed over ranks (max time over ranks).
    gguf: the model of that GGUF file instead (its weights uploaded once and
    shared by the batch sizes)."""
    import torch

    from swq.model import LlamaConfig, LlamaDecoder

    need = prefill + steps + warmup + 8
    W = None
    if gguf is None:
        cfg = LlamaConfig(max_seq=need)
        model = "Llama-3-8B shape, Q4_K_M mix (Q6_K attn_v/ffn_down/output, Q4_K else), synthetic weights"
    else:
        from swq.gguf import llama_from_gguf
        cfg, W, _file = llama_from_gguf(gguf, context_override=need)
        if cfg.max_seq < need:
            raise ValueError(f"{gguf}: context {cfg.max_seq} < the {need} positions this run needs")
        model = f"GGUF file {os.path.basename(gguf)} ({cfg.n_layers} layers, hidden {cfg.dim}, vocab {cfg.vocab})"
    out = {"model": model, "context": prefill, "steps": steps,
           "weight_bytes_per_token": cfg.weight_bytes_per_token(), "batches": {}}
    dist = None
    if world > 1:
        import torch.distributed as dist
    first = None
    for B in batches:
        log(f"decode8b: batch {B} (one model per rank)")
        if gguf is None:
            dec = LlamaDecoder(cfg, rows=B, seed=100 + rank)
        else:
            dec = LlamaDecoder(cfg, rows=B, weights=None if first else W, weights_from=first)
            first = first or dec
        dec.reset(list(range(B)), 0)
        dec.capture()
        ctx = _build_context(dec, prefill, seed=11)
        dec.generate(warmup)
        dec.stream.synchronize()
        if dist:
            dist.barrier()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(dec.stream)
        dec.generate(steps)
        ev1.record(dec.stream)
        ev1.synchronize()
        ms = ev0.elapsed_time(ev1)
        if dist:
            t = torch.tensor([ms], dtype=torch.float64, device=dec.device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        ok = bool(torch.isfinite(dec.logits).all().item())
        per_tok_ms = ms / steps
        out["batches"][str(B)] = {
            "tok_s": round(B * steps * world / (ms * 1e-3), 1), "ms_per_step": round(per_tok_ms, 4),
            "weight_GBps": round(cfg.weight_bytes_per_token() / (per_tok_ms * 1e-3) / 1e9, 1),
            "finite_logits": ok, **ctx}
        if dec is not first:
            del dec
            torch.cuda.empty_cache()
    return out


def run_decode_moe(rank: int, world: int, B: int = 32, prefill: int = 1024, steps: int = 64,
                   warmup: int = 4) -> dict:
    """The MoE decoder (40 layers, hidden 2048, 16/4 heads of 128, 256 experts
    of 512 top-8 + a shared expert of 512, Q4_K experts, vocab 151936,
    synthetic weights generated on the device), experts sharded over the
    ranks and each rank decoding its own rows with the whole attention: a
    `prefill`-token prompt prefilled at batch 1 (timed), then `B` rows sharing
    its K/V decode `steps` graph-replayed greedy steps.  tok/s of all ranks
    (max time over ranks)."""
    import numpy as np
    import torch

    from swq.model import LlamaConfig, LlamaDecoder

    cfg = LlamaConfig.moe_40l(max_seq=prefill + steps + warmup + 8)
    dist = None
    if world > 1:
        import torch.distributed as dist
    grp = dist.group.WORLD if dist else None
    log(f"decode_moe: building (experts over {world} ranks)")
    one = LlamaDecoder(cfg, rows=1, seed=3, ep_group=grp, moe_max_tokens=prefill)
    toks = [((np.arange(prefill) * 7919 + 13 * rank) % cfg.vocab).tolist()]
    one.prefill(toks)  # warm-up of the prefill path (same calls on every rank)
    one.stream.synchronize()
    if dist:
        dist.barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(one.stream)
    one.prefill(toks)
    ev1.record(one.stream)
    ev1.synchronize()
    pf_ms = ev0.elapsed_time(ev1)
    dec = LlamaDecoder(cfg, rows=B, weights_from=one)
    dec.reset(list(range(B)), 0)
    dec.capture()
    ctx = _build_context(dec, prefill, seed=5, share_from=one)
    dec.generate(warmup)
    dec.stream.synchronize()
    if dist:
        dist.barrier()
    ev0.record(dec.stream)
    dec.generate(steps)
    ev1.record(dec.stream)
    ev1.synchronize()
    ms = ev0.elapsed_time(ev1)
    if dist:
        t = torch.tensor([ms, pf_ms], dtype=torch.float64, device=dec.device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, pf_ms = float(t[0].item()), float(t[1].item())
    import swq
    swq.check(dec.stream)
    ok = bool(torch.isfinite(dec.logits).all().item())
    out = {"model": "MoE decoder: 40 layers, hidden 2048, 16/4 heads of 128, 256 experts x 512 top-8 + shared 512, "
                    "Q4_K experts, vocab 151936, synthetic weights", "expert_parallel": world,
           "prefill": {"tokens_per_rank": prefill, "ms": round(pf_ms, 2),
                       "tok_s": round(world * prefill / (pf_ms * 1e-3), 1)},
           "decode": {"batch_per_rank": B, "steps": steps, "ms_per_step": round(ms / steps, 3),
                      "tok_s": round(world * B * steps / (ms * 1e-3), 1), "finite_logits": ok, **ctx}}
    dec.graph = None
    del dec, one
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return out


def run_decode_tp(rank: int, world: int, batches=(1, 8, 32), context: int = 2048, steps: int = 32,
                  warmup: int = 4, collective: str = "peer") -> dict:
    """Greedy decode of a Llama-3-70B-shaped model (80 layers, hidden 8192,
    64/8 heads of 128, FFN 28672, vocab 128256, Q4_K_M mix, synthetic weights
    generated on the device), tensor-parallel over all ranks (column-sharded
    q/k/v and gate/up, row-sharded o and down with an NCCL all-reduce each,
    vocab-sharded LM head with an all-gather), after a `context`-token prefill
    of uniform random token ids (batch 1, timed on its own; the larger batches
    share that prompt's K/V).  One rank: the whole model on one GPU.  tok/s =
    tokens of the whole job per second (max time over ranks)."""
    import torch

    from swq.model import LlamaConfig, LlamaDecoder

    cfg = LlamaConfig.llama3_70b(max_seq=context + steps + warmup + 8)
    wbytes = cfg.weight_bytes_per_token()
    sums = ("one-shot all-reduce over NVLink peer memory (libswq)" if collective == "peer"
            else "NCCL all-reduce")
    out = {"model": "Llama-3-70B shape, Q4_K_M mix, synthetic weights", "tensor_parallel": world,
           "context": context, "steps": steps, "weight_bytes_per_token": wbytes,
           "collectives": f"{sums} after o and down, NCCL all-gather of the logits, in the CUDA graph"
           if world > 1 else "none", "batches": {}}
    dist = None
    if world > 1:
        import torch.distributed as dist
    base = None
    for B in batches:
        log(f"decode70b: tp={world} batch {B}: building")
        dec = LlamaDecoder(cfg, rows=B, seed=7, weights_from=base, collective=collective,
                           group=dist.group.WORLD if dist else None)
        base = base or dec
        dec.reset(list(range(B)), 0)
        dec.capture()
        import swq
        swq.check(dec.stream)  # a collective that timed out fails here, not in the timed loop
        log(f"decode70b: tp={world} batch {B}: captured")
        # the same prompt on every rank; batches above 1 share the batch-1 prefill
        ctx = _build_context(dec, context, seed=13,
                             share_from=base if (dec is not base and DECODE_CONTEXT == "prefill") else None)
        dec.generate(warmup)
        dec.stream.synchronize()
        swq.check(dec.stream)
        if dist:
            dist.barrier()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(dec.stream)
        dec.generate(steps)
        ev1.record(dec.stream)
        ev1.synchronize()
        ms = ev0.elapsed_time(ev1)
        if dist:
            t = torch.tensor([ms], dtype=torch.float64, device=dec.device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        ok = bool(torch.isfinite(dec.logits).all().item())
        per_step = ms / steps
        out["batches"][str(B)] = {
            "tok_s": round(B * steps / (ms * 1e-3), 1), "ms_per_step": round(per_step, 3),
            "weight_GBps_per_gpu": round(wbytes / world / (per_step * 1e-3) / 1e9, 1),
            "finite_logits": ok, **ctx}
        dec.graph = None  # release the graph (it holds NCCL calls) before the next one
        if dec is not base:
            del dec
        torch.cuda.synchronize()
    base.graph = None
    del base
    torch.cuda.empty_cache()
    return out


# ---------------------------------------------------------------- config-1 sweep
SWEEP_FORMATS = ("Q4_0", "Q8_0", "Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K")
SWEEP_MS = (1, 8, 64, 512)


def run_sweep(N: int = 14336, K: int = 4096, launches: int = 40, cpu_seconds: float = 1.0) -> dict:
    """Quant-format x batch sweep on the Llama-3-8B FFN up-projection shape:
    Y[M x N] = X[M x K] . W^T for every format and M in SWEEP_MS, through
    swq_gemm (the fused GEMV kernel for M < 5, the tensor-core GEMM above),
    CUDA-event timed over `launches` calls that rotate over weight copies
    larger than 4 x L2 together.  Roofline per point: HBM (weight + X + Y
    bytes) and tensor (2 M N K flops), whichever bounds it.  Beside each, the
    reference's CPU routine on all host cores: one matmul_transposed_q per
    activation row (it has no batched path), its per-row time measured on a
    bounded sample and multiplied by M."""
    import torch

    import oracle
    import swq
    from swq import synth
    from swq.model import synthetic_blocks

    dev = torch.device("cuda", torch.cuda.current_device())
    hbm, hbm_kind = load_peaks()
    tc, tc_kind = load_tensor_peak()
    g = torch.Generator(device=dev)
    g.manual_seed(41)
    cores = oracle.host_cores()
    use_ref = oracle.ref_available()
    (oracle.ref_set_threads if use_ref else oracle.set_threads)(cores)
    out = {"shape": f"N={N} K={K}", "launches_per_point": launches,
           "peaks": {"hbm_GBps": hbm, "hbm_kind": hbm_kind, "bf16_TFLOPs": tc, "tensor_kind": tc_kind},
           "cpu": {"kind": "reference" if use_ref else "port", "cores": cores,
                   "sample": f"matmul_transposed_q on {cores} threads, about {cpu_seconds:.1f} s per format; "
                             "M > 1 is M such calls"},
           "points": []}
    for name in SWEEP_FORMATS:
        t = TYPE_IDS[name]
        wbytes = synth.matrix_bytes(t, N, K)
        copies = max(2, -(-4 * 126_000_000 // wbytes))
        ws = [synthetic_blocks(t, N, K, g, dev) for _ in range(copies)]
        # the reference's per-row time: one host matrix, rows of X cycled
        hw = synth.fast_random_blocks(t, N, K, seed=90 + t)
        hx = synth.random_activations(4, K, seed=91)
        fn = (lambda w, x: oracle.ref_gemv(t, w, x, N, K)) if use_ref else \
             (lambda w, x: oracle.gemv(t, w, x, N, K))
        fn(hw, hx[0])
        n, t0 = 0, time.perf_counter()
        while True:
            fn(hw, hx[n % 4])
            n += 1
            if time.perf_counter() - t0 >= cpu_seconds:
                break
        cpu_row_s = (time.perf_counter() - t0) / n
        for M in SWEEP_MS:
            X = torch.randn((M, K), device=dev, generator=g)
            Y = torch.empty((M, N), device=dev)
            for i in range(3):
                swq.gemm(t, ws[i % copies], X, Y, M, N, K)
            swq.check()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for i in range(launches):
                swq.gemm(t, ws[i % copies], X, Y, M, N, K)
            e1.record()
            e1.synchronize()
            swq.check()
            sec = e0.elapsed_time(e1) * 1e-3 / launches
            nbytes = wbytes + 4 * M * K + 4 * M * N
            flops = 2.0 * M * N * K
            gbs, tfs = nbytes / sec / 1e9, flops / sec / 1e12
            tc_path = M >= swq.get_option(swq.OPT_TENSOR_CORE_MIN_M) and not _batched_path(name, M)
            t_roof = max(nbytes / (hbm * 1e9), flops / (tc * 1e12))
            out["points"].append({
                "format": name, "M": M, "us": round(sec * 1e6, 2), "GBps": round(gbs, 1), "TFLOPs": round(tfs, 2),
                "path": "tensor-core GEMM (fp16 operands, fp32 accumulate)" if tc_path else _gemv_form(name, M),
                "bound": "tensor" if flops / (tc * 1e12) > nbytes / (hbm * 1e9) else "hbm",
                "roofline_frac": round(t_roof / sec, 4),
                "cpu_ms": round(cpu_row_s * M * 1e3, 3), "speedup_vs_cpu": round(cpu_row_s * M / sec, 1)})
        del ws
        torch.cuda.empty_cache()
    return out


# ---------------------------------------------------------------- MoE workload
def run_moe(rank: int, world: int, steps: int = 20, warmup: int = 3) -> dict:
    """One MoE FFN layer of the MoE decoder shape (hidden 2048; 256 routed
    experts of intermediate 512 with gate, up, down in Q4_K, synthetic blocks
    generated on the device; one shared expert of 512; fp32 router N(0, 0.02),
    top-8 softmax routing), experts sharded over the ranks (256/G each), every
    step on the device (swq.moe.MoEFFN: router and top-k kernels, peer-memory
    dispatch and combine, grouped expert GEMMs).  Each rank routes its own
    tokens: a 1024-token prefill and a batch of 32 decode tokens per rank.
    Reported per case, max over ranks, CUDA events:
      grouped: the expert GEMMs alone (gate|up, SiLU-mul, down) on the rows
        this rank received, against their weight-stream floor (the bytes of
        the experts that received rows / measured HBM copy bandwidth);
      exchange: dispatch + combine alone (rows to the experts' ranks over
        NVLink and the outputs back), with the bytes that cross NVLink;
      layer: the whole layer captured in a CUDA graph, tokens/s of all ranks."""
    import numpy as np
    import torch

    import swq
    from swq.model import synthetic_blocks
    from swq.moe import MoEFFN
    from swq.synth import row_bytes

    dev = torch.device("cuda", torch.cuda.current_device())
    E, H, F, k, Fs = 256, 2048, 512, 8, 512
    t = swq.Q4_K
    if E % world:
        return {"skipped": f"{E} experts do not split over {world} ranks"}
    el = E // world
    g = torch.Generator(device=dev)
    g.manual_seed(31 + rank)
    gu_all = synthetic_blocks(t, el * 2 * F, H, g, dev)
    d_all = synthetic_blocks(t, el * H, F, g, dev)
    gr = torch.Generator(device=dev)
    gr.manual_seed(5)  # the router and the shared expert are the same on every rank
    router = torch.randn(E, H, generator=gr, device=dev) * 0.02
    shared = (synthetic_blocks(t, Fs, H, gr, dev), synthetic_blocks(t, Fs, H, gr, dev),
              synthetic_blocks(t, H, Fs, gr, dev))
    expert_bytes = 2 * F * row_bytes(t, H) + H * row_bytes(t, F)
    dist = None
    if world > 1:
        import torch.distributed as dist
    peak, _ = load_peaks()
    out = {"model": "MoE FFN: hidden 2048, 256 experts x (gate, up 512x2048; down 2048x512) Q4_K + 1 shared "
                    "expert of 512, fp32 router, top-8", "expert_parallel": world, "experts_per_rank": el,
           "expert_bytes": expert_bytes, "tokens_per_rank": {"prefill": 1024, "decode": 32},
           "exchange": "peer-memory dispatch/combine (swq_ep_*), counts exchanged on the device"}

    def timed(fn, n):
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n):
            fn()
        e1.record()
        e1.synchronize()
        ms = e0.elapsed_time(e1) / n
        if dist:
            tt = torch.tensor([ms], dtype=torch.float64, device=dev)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            ms = float(tt.item())
        return ms

    def max_over_ranks(v):
        if not dist:
            return v
        tt = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        return float(tt.item())

    base = None
    for name, T in (("prefill_1024", 1024), ("decode_32", 32)):
        moe = MoEFFN(None, (t, t, t), H, F, router, k, max_tokens=T, group=dist.group.WORLD if dist else None,
                     device=dev, shared=shared, shared_types=(t, t, t), shared_F=Fs, n_experts=E,
                     device_blocks=(gu_all, d_all))
        x = torch.randn(T, H, generator=g, device=dev)
        for _ in range(warmup):
            moe(x, T)
        swq.check()
        # which experts got rows here, from this call's routing (outside the timing)
        moe.route(x, T)
        ids_all = [moe.ids[:T].clone()]
        if dist:
            gathered = [torch.empty_like(ids_all[0]) for _ in range(world)]
            dist.all_gather(gathered, ids_all[0])
            ids_all = gathered
        ids_np = np.concatenate([i.cpu().numpy().reshape(-1) for i in ids_all])
        mine = ids_np[(ids_np >= rank * el) & (ids_np < (rank + 1) * el)]
        touched = int(np.unique(mine).size)
        rows = int(mine.size)
        moe.ep.dispatch(x, moe.ids, T)
        ms_g = timed(lambda: moe.experts(T, peer_tokens=T), steps)
        floor_ms = touched * expert_bytes / (peak * 1e9) * 1e3
        ms_g_floor = max_over_ranks(floor_ms)

        def exchange():
            moe.ep.dispatch(x, moe.ids, T)
            moe.ep.combine(moe.y_recv, moe.w, moe.y)

        ms_x = timed(exchange, steps)
        remote = int(((ids_np // el) != np.repeat(np.arange(world), T * k)).sum()) if world > 1 else 0
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            moe(x, T, peer_tokens=T, stream=s)
        s.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            moe(x, T, peer_tokens=T, stream=s)
        ms_l = timed(graph.replay, steps)
        swq.check()
        del graph
        out[name] = {
            "grouped": {"ms": round(ms_g, 4), "rows_this_rank": rows, "experts_touched_this_rank": touched,
                        "weight_GBps": round(touched * expert_bytes / (ms_g * 1e-3) / 1e9, 1),
                        "floor_ms": round(ms_g_floor, 4), "frac_of_floor": round(ms_g_floor / ms_g, 3),
                        "tflops": round(2.0 * rows * 3 * F * H / (ms_g * 1e-3) / 1e12, 2)},
            "exchange": {"ms": round(ms_x, 4), "rows_over_nvlink_all_ranks": remote,
                         "bytes_over_nvlink_all_ranks": remote * H * 4 * 2},
            "layer": {"ms": round(ms_l, 4), "tok_s": round(world * T / (ms_l * 1e-3), 1)},
        }
        moe.ep.close()
        del moe
        torch.cuda.synchronize()
    out["hbm_peak_GBps"] = peak
    return out


# ---------------------------------------------------------------- GEMM workload
GEMM_N, GEMM_K = 14336, 4096
TYPE_IDS = {"Q4_0": 2, "Q8_0": 8, "Q2_K": 10, "Q3_K": 11, "Q4_K": 12, "Q5_K": 13, "Q6_K": 14}
# dram__bytes_read.sum + dram__bytes_write.sum of one gemm_kernel launch, Q4_K
# N=14336 K=4096 M=512, from one ncu capture (profiles/gemm_q4k_14336x4096_m512.md).
NCU_TRAFFIC_GEMM_Q4K_M512 = 37_271_552 + 1_266_944


def cpu_gemm_timing(type_id: int, M: int, seconds: float, N: int = GEMM_N, K: int = GEMM_K) -> dict | None:
    """The reference's prefill: one Compute::matmul_transposed_q per token, on
    all host cores.  A bounded sample of tokens; TFLOP/s of the rows done."""
    import oracle
    from swq import synth
    if seconds <= 0:
        return None
    cores = oracle.host_cores()
    if oracle.ref_available():
        kind = "reference"
        oracle.ref_set_threads(cores)
        fn = lambda w, x: oracle.ref_gemv(type_id, w, x, N, K)  # noqa: E731
    else:
        kind = "port"
        oracle.set_threads(cores)
        fn = lambda w, x: oracle.gemv(type_id, w, x, N, K, format_order=False)  # noqa: E731
    w = synth.random_blocks(type_id, N, K, seed=77)
    X = synth.random_activations(min(M, 64), K, seed=78)
    fn(w, X[0])
    n = 0
    t0 = time.perf_counter()
    while True:
        fn(w, X[n % X.shape[0]])
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds or n >= M:
            break
    tf = 2.0 * N * K * n / el / 1e12
    return {"value": round(tf, 5), "unit": "TFLOP/s", "cores": cores, "kind": kind,
            "sample": f"{n} of the M={M} token rows (one matmul_transposed_q each), {el:.1f} s, "
                      f"{cores} OpenMP threads"}


def run_gemm(args, rank: int, world: int) -> None:
    import numpy as np
    import torch

    import swq
    from swq import synth

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    t = TYPE_IDS[args.format]
    M, N, K = args.M, args.N, args.K
    wbytes = synth.matrix_bytes(t, N, K)
    copies = max(2, -(-4 * 126_000_000 // wbytes))
    host_ws = [synth.random_blocks(t, N, K, seed=20_000 + i) for i in range(copies)]
    d_ws = [torch.from_numpy(w.reshape(-1)).to(dev) for w in host_ws]
    X = synth.random_activations(M, K, seed=21)
    d_x = torch.from_numpy(X).to(dev)
    d_y = torch.empty((M, N), dtype=torch.float32, device=dev)
    stream = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(stream):
        for i in range(max(3, args.warmup)):
            swq.gemm(t, d_ws[i % copies], d_x, d_y, M, N, K, stream=stream)
    swq.check(stream)
    gpu_uuid = str(torch.cuda.get_device_properties(dev).uuid)
    gpu_uuid = gpu_uuid if gpu_uuid.startswith("GPU-") else f"GPU-{gpu_uuid}"
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(gpu_uuid) as clk:
        with torch.cuda.stream(stream):
            ev0.record(stream)
            for i in range(args.steps):
                swq.gemm(t, d_ws[i % copies], d_x, d_y, M, N, K, stream=stream)
            ev1.record(stream)
        ev1.synchronize()
    ms = ev0.elapsed_time(ev1)
    swq.check(stream)
    flops = 2.0 * M * N * K
    per_call_s = ms * 1e-3 / args.steps
    value = flops * world / per_call_s / 1e12
    peak, peak_kind = load_tensor_peak()
    hbm_peak, hbm_kind = load_peaks()
    tc_path = M >= swq.get_option(swq.OPT_TENSOR_CORE_MIN_M) and not _batched_path(args.format, M)

    # End to end through the host-buffer API: host X in, host Y out.
    comp = swq.Compute(device=local)
    Y = np.zeros((M, N), np.float32)
    qw = swq.QuantWeight(host_ws[0], t)
    comp.matmul_q_batched(Y, X, qw, M, N, K)  # weights uploaded once
    e2e_steps = max(1, min(args.steps, 50))
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        comp.matmul_q_batched(Y, X, qw, M, N, K)
    e2e_s = time.perf_counter() - t0
    comp.close()
    if rank != 0:
        return
    line = {
        "metric": f"dequant-GEMM TFLOP/s (N={N} K={K})", "value": round(value, 1),
        "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms / args.steps, 5), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None,
        "dtype": ("f16 operands, f32 accumulate" if tc_path else
                  "f32 (x as fp16 pairs per super-block, exact products, fp32 sums)"
                  if _batched_path(args.format, M) else "f32"),
        "data": "synthetic",
        "config": {"workload": f"{args.format} dequant-GEMM M={M} N={N} K={K}, {copies} rotating weight copies",
                   "format": args.format, "M": M, "N": N, "K": K, "copies": copies,
                   "l2": "inputs larger than L2 (rotating weights)"},
        "roofline": ({"bound": "tensor", "achieved": round(flops / per_call_s / 1e12, 1), "peak": peak,
                      "unit": "TFLOP/s", "frac": round(flops / per_call_s / 1e12 / peak, 4),
                      "peak_kind": peak_kind,
                      "traffic": NCU_TRAFFIC_GEMM_Q4K_M512 if (args.format, M) == ("Q4_K", 512) else None,
                      "kernel": "swq::tc::gemm_kernel (+ x_to_f16_kernel)",
                      "us_per_call": round(per_call_s * 1e6, 2)} if tc_path else
                     {"bound": "hbm", "achieved": round(wbytes / per_call_s / 1e9, 1), "peak": hbm_peak,
                      "unit": "GB/s", "frac": round(wbytes / per_call_s / 1e9 / hbm_peak, 4),
                      "peak_kind": hbm_kind, "traffic": None, "kernel": _gemv_form(args.format, M),
                      "us_per_call": round(per_call_s * 1e6, 2)}),
        "cpu_baseline": cpu_gemm_timing(t, M, args.cpu_seconds, N, K) if world == 1 else None,
        "e2e": {"value": round(flops * e2e_steps / e2e_s / 1e12, 2), "unit": "TFLOP/s",
                "h2d_bytes_per_step": 4 * M * K, "d2h_bytes_per_step": 4 * M * N,
                "api": "swq_ctx_matmul_q_batched (host fp32 X/Y, resident weights)", "steps": e2e_steps},
        "gpu_launches": (2 if tc_path else 1) * args.steps,
        "clocks": clk.summary(),
        "weight_GBps": round(wbytes / per_call_s / 1e9, 1),
    }
    emit(line)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20,
                    help="timed steps (headline: a step is 128 replays of the 64-GEMV graph)")
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["swq", "reference"], default="swq")
    ap.add_argument("--workload", choices=["gemv", "gemm", "decode", "decode70b", "moe", "prefill", "prefill70b"],
                    default="gemv",
                    help="gemv: the headline Q4_K GEMV (with decode tok/s); gemm: the prefill dequant-GEMM; "
                         "decode: Llama-3-8B greedy decode tok/s alone (replicas); decode70b: Llama-3-70B "
                         "decode tok/s, tensor-parallel over the ranks; prefill / prefill70b: batched prefill "
                         "of one prompt (--M tokens, default 512) on one GPU")
    ap.add_argument("--format", choices=sorted(TYPE_IDS), default="Q4_K", help="GEMM weight format")
    ap.add_argument("--M", type=int, default=512, help="GEMM activation rows (below 5: the GEMV kernel)")
    ap.add_argument("--N", type=int, default=GEMM_N, help="GEMM weight rows")
    ap.add_argument("--K", type=int, default=GEMM_K, help="GEMM weight columns")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="CPU sample length (0: skip)")
    ap.add_argument("--collective", choices=["peer", "nccl"], default="peer",
                    help="decode70b: sums of the row-parallel projections")
    ap.add_argument("--no-sweep", dest="sweep", action="store_false",
                    help="skip the quant-format x batch sweep (N=14336, K=4096) of the default one-GPU run")
    ap.add_argument("--no-moe", dest="moe", action="store_false",
                    help="skip the MoE layer measurement (config 3 shape) of the default run")
    ap.add_argument("--no-decode", dest="decode", action="store_false",
                    help="skip the Llama-3-8B decode tok/s measurement of the default run")
    ap.add_argument("--gguf", default=None, help="--workload decode: decode this GGUF model file instead of "
                                                  "the synthetic Llama-3-8B-shaped one")
    ap.add_argument("--prefill-attention", type=int, choices=[0, 1, 2, 3], default=None,
                    help="--workload prefill|prefill70b: SWQ_OPT_PREFILL_ATTENTION for the run (default: the "
                         "library's, 3)")
    ap.add_argument("--decode-context", choices=["synthetic", "prefill"], default="prefill",
                    help="decode measurements: context as random K/V (synthetic) or a batched prefill of "
                         "random prompt tokens (prefill, also timed)")
    args = ap.parse_args()
    _claim_stdout()
    global DECODE_CONTEXT
    DECODE_CONTEXT = args.decode_context
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if args.warmup < 3:
        log("warm-up raised to 3 steps (minimum)")
        args.warmup = 3
    if args.workload == "moe":
        import torch
        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        if world > 1:
            import datetime

            import torch.distributed as dist
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                    device_id=torch.device("cuda", local))
        d = run_moe(rank, world, steps=args.steps if args.steps != ap.get_default("steps") else 20)
        if args.decode:
            d["decoder"] = run_decode_moe(rank, world)
        if rank == 0:
            lay = d.get("decode_32", {}).get("layer", {})
            emit({"metric": "MoE layer tok/s (decode batch 32 per GPU, 256 experts top-8, Q4_K)",
                  "value": lay.get("tok_s"), "unit": "tok/s", "n_gpus": world,
                  "higher_is_better": True, "scaling": "weak", "data": "synthetic", "moe": d})
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return
    if args.workload in ("prefill", "prefill70b"):
        import torch
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        if world > 1 and rank == 0:
            log("prefill runs on one GPU; other ranks exit")
        if rank != 0:
            return
        if args.prefill_attention is not None:
            import swq
            swq.set_option(swq.OPT_PREFILL_ATTENTION, args.prefill_attention)
        d = run_prefill(rank, prompt=args.M, seventy=args.workload == "prefill70b")
        emit({"metric": f"prefill tok/s ({d['model']}, {args.M}-token prompt)", "value": d["tok_s"],
              "unit": "tok/s", "n_gpus": 1, "higher_is_better": True, "data": "synthetic",
              "prefill": d})
        return
    if args.workload in ("decode", "decode70b"):
        import torch
        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        if world > 1:
            import datetime

            import torch.distributed as dist
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                    device_id=torch.device("cuda", local))
        if args.workload == "decode":
            d = run_decode(rank, world, steps=args.steps if args.steps != ap.get_default("steps") else 256,
                           gguf=args.gguf)
            name = f"decode tok/s ({'Llama-3-8B Q4_K_M' if args.gguf is None else d['model']}, batch 1)"
            scaling = "weak"
        else:
            d = run_decode_tp(rank, world, steps=args.steps if args.steps != ap.get_default("steps") else 32,
                              collective=args.collective)
            name, scaling = f"decode tok/s (Llama-3-70B Q4_K_M, batch 1, tensor-parallel x{world})", "strong"
        if rank == 0:
            b1 = d["batches"]["1"]
            emit({"metric": name, "value": b1["tok_s"],
                  "unit": "tok/s", "n_gpus": world, "higher_is_better": True, "scaling": scaling,
                  "data": "synthetic", "decode": d})
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return
    if args.workload == "gemm":
        if args.steps == ap.get_default("steps"):
            args.steps = 2000
        run_gemm(args, rank, world)
        return
    run_swq(args, rank, world)


if __name__ == "__main__":
    main()
