#!/usr/bin/env python
"""Benchmark of the B200 row-op hot path (libtb_b200.so), one JSON line.

Default workload (--config 70b): one pass of the per-token row ops of a
Llama-3-70B-shape prefill of 16384 tokens (8 sequences x 2048), strong-
scaled: the token rows, the logit rows and the embedding table's vocabulary
rows are split over the N ranks (tb_b200_partition).
  embedding gather          16384 ids -> rows of a [128256, 8192] bf16 table,
                            vocab-sharded: each rank holds 128256/N table
                            rows in NCCL symmetric memory and gathers its
                            token part in one kernel that loads rows from
                            the owners' windows
                            (tb_b200_embedding_sharded_window); the NCCL
                            send/recv exchange and the CUDA IPC gather are
                            timed beside the step
  residual + RMSNorm        [16384/N, 8192]                   } one fused
  RoPE on Q and K           [16384/N, 64 | 8, 128], pos % 2048 } layer-chain
  SwiGLU silu(gate)*up      [16384/N, 28672]                   } launch
  row softmax               logits [4096/N, 128256] f32
  greedy argmax             logits [4096/N, 128256] f32 (own buffer)
--config 7b is the Llama-7B prefill of 4096 tokens (embedding from a
[32000, 4096] table, chain, softmax/argmax over [4096, 32000]) run whole on
every rank (weak scaling).  Activations bf16 (f32 arithmetic), logits f32;
synthetic seeded inputs with the reference configs' distributions.  Every
op reads distinct buffers and a step moves GBs, far more than the 126 MB L2.

metric: algorithmic HBM bytes of the step (each input read once, each
output written once) over all ranks / device time (max over ranks), in
GB/s; rows/s beside it.

--impl reference times the reference's own CPU kernels (oracle/_ref, the
reference's src/ops/*.c) on the host's cores over a bounded row sample of
the same workload.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "tensorbit-run_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import workloads as W  # noqa: E402

# --config: the default (70b) is the Llama-70B prefill's row ops on 16384
# tokens with softmax/argmax over 4096 rows of 128256 logits, strong-scaled
# over the ranks; 7b is the Llama-7B prefill of 4096 tokens on every rank.
CONFIGS = {
    "7b": (W.CONFIGS["7b"], None, "llama7b-prefill-4096 row ops (embedding, residual+RMSNorm, "
                                  "RoPE, SwiGLU, softmax, argmax)"),
    "70b": (W.CONFIGS["70b"], 4096, "llama70b-prefill-16384 (8 x 2048) row ops strong-scaled "
                                    "over the ranks: vocab-sharded 128256 x 8192 embedding "
                                    "gather (one kernel over the NCCL symmetric-memory "
                                    "windows), residual+RMSNorm, RoPE, SwiGLU, "
                                    "softmax/argmax over 4096 x 128256 logits"),
    "sweep": (W.CONFIGS["7b"], None, "bandwidth sweep: residual+RMSNorm and SwiGLU over rows "
                                     "2^10..2^20 x hidden {2048, 4096, 8192, 16384} in f32 and "
                                     "bf16; softmax and argmax over rows {1, 16, 256, 4096} x "
                                     "128256 f32 logits; rows split over the ranks"),
    "decode": (W.CONFIGS["decode"], None, "decode 256 sequences x 1 token at the llama7b shape: the "
                                          "fused layer chain (residual+RMSNorm, RoPE, SwiGLU) over "
                                          "32 layers, one CUDA graph"),
    "runner": (W.CONFIGS["7b"], None, "TransformerRunner decode of one sequence at the llama7b "
                                      "shape (32 layers, f32 weights, 2:4-pruned projections), "
                                      "one CUDA graph per token"),
    "runner_int4": (W.CONFIGS["7b"], None, "TransformerRunner decode of one sequence at the llama7b "
                                           "shape (32 layers, INT4 projections in groups of 128, "
                                           "f32 embedding and lm head), one CUDA graph per token"),
}
RUNNER_GROUP = 128  # INT4 scale group of --config runner_int4
RUNNER_LAYERS = 32
RUNNER_MAX_SEQ = 2048
RUNNER_CONTEXT = 1024  # tokens fed (untimed) before the timed ones: decode at context 1024+
RUNNER_METRIC = "decode tokens/s"
DECODE_LAYERS = 32
DEFAULT_CONFIG = "70b"
CFG, LOGIT_ROWS, WORKLOAD = CONFIGS[DEFAULT_CONFIG]
SEQ_LEN_70B = 2048  # the 70b prefill's 16384 tokens are 8 sequences of 2048
TABLE_CHUNK = 4096  # embedding-table rows drawn per seed (rank-count independent)
E2E_BLOCKS = 8    # row blocks of the end-to-end step
E2E_STREAMS = 3   # streams they are spread over
METRIC = "fused layer-op HBM GB/s"


def logit_rows(rows):
    """Rows of the softmax/argmax logits for `rows` layer-op rows."""
    return rows if LOGIT_ROWS is None else min(rows, LOGIT_ROWS)


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per row of each
# kernel, from one ncu capture of that kernel at the config's row shape, for
# roofline.traffic.  Writes still dirty in L2 when a kernel ends are not in
# the write count.
TRAFFIC_PER_ROW = {
    "7b": {
        "embedding": 32137856 / 4096,
        "layer_chain": 485573888 / 4096,
        "softmax": (200159488 + 75085568) / 1024,
        "argmax": 530358016 / 4096,
    },
    # captured on one GPU: softmax/argmax over 1024 x 128256 logits, the
    # layer chain over 2048 token rows, the gather of 8192 tokens
    "70b": {
        "embedding": (130690304 + 84914432) / 8192,
        "layer_chain": (340854784 + 167031552) / 2048,
        "softmax": (1178672384 + 467714048) / 1024,
        "argmax": (525479680 + 4182784) / 1024,
    },
}
# What bounds each op of the 70b step, for the line's "limiter".
LIMITER_NOTE = {
    "softmax": "the in-order row sum reads the row three times; two 501 KB rows per SM in "
               "flight are a little more than the L2 holds, so DRAM moves ~1.6x the "
               "algorithmic bytes, and the per-tile reduction chains bound the issue rate",
    "layer_chain": "HBM bandwidth (~0.9 of the copy peak)",
    "argmax": "HBM bandwidth (read-only stream at the copy peak)",
    "embedding": "HBM on one GPU; NVLink peer reads with more GPUs",
}
TRAFFIC_SOURCE = "ncu capture of the kernel (DRAM bytes read + written per row, scaled to the " \
                 "launch's rows)"


def step_bytes(rows, act_s, lr=None):
    c = CFG
    lr = logit_rows(rows) if lr is None else lr
    parts = {
        "embedding": W.bytes_embedding(rows, c.hidden, act_s),
        "layer_chain": (W.bytes_res_rms(rows, c.hidden, act_s)
                        + W.bytes_rope(rows, c.n_q_heads, c.n_kv_heads, c.head_dim, act_s)
                        + W.bytes_swiglu(rows, c.intermediate, act_s)),
        "softmax": W.bytes_softmax(lr, c.vocab, 4),
        "argmax": W.bytes_argmax(lr, c.vocab, 4),
    }
    return parts


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """Samples SM clock and clock-event reasons with NVML while running."""
    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
               0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}

    def __init__(self, index, uuid=None):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        try:
            import pynvml as N
            N.nvmlInit()
            self.N = N
            self.h = None
            if uuid:
                try:
                    self.h = N.nvmlDeviceGetHandleByUUID(uuid)
                except Exception:
                    self.h = None
            if self.h is None:
                self.h = N.nvmlDeviceGetHandleByIndex(index)
            self.get_reasons = getattr(N, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                N.nvmlDeviceGetCurrentClocksThrottleReasons
            self.max_mhz = N.nvmlDeviceGetMaxClockInfo(self.h, N.NVML_CLOCK_SM)
        except Exception as e:  # no NVML: report it, do not guess
            self.N, self.err = None, str(e)

    def _run(self):
        N = self.N
        while not self._stop.is_set():
            try:
                self.samples.append(N.nvmlDeviceGetClockInfo(self.h, N.NVML_CLOCK_SM))
                bits = self.get_reasons(self.h)
                for b, name in self.REASONS.items():
                    if bits & b:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.005)

    def __enter__(self):
        if self.N:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self.N:
            self.t.join()

    def summary(self):
        if not self.N:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "error": self.err}
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons - {"gpu_idle"}),
                "samples": len(self.samples)}


# ------------------------------------------------------------- CPU baseline
def cpu_sample(rows=256):
    """One pass of the step over `rows` rows of every op, on the host cores,
    through the reference's own kernels (oracle/_ref; the restatement if the
    reference build is absent).  Returns (run, bytes, kind, cores)."""
    import numpy as np
    from oracle import oracle as O
    O.lib()
    impl, kind = (O.REF, "reference") if O.ref_available() else (O.PORT, "port")
    cores = os.cpu_count() or 1
    c = CFG
    li = W.layer_inputs(c, rows=rows)
    bf = O.f32_to_bf16
    x, res, gam = bf(li["x"]), bf(li["res"]), bf(li["gamma"])
    q, k = bf(li["q"]), bf(li["k"])
    gate, up = bf(li["gate"]), bf(li["up"])
    rng = np.random.default_rng(c.seed + 7)
    vt = min(c.vocab, 32768)  # table rows of the host sample (the gather's cost is per row)
    table = bf(rng.standard_normal((vt, c.hidden), dtype=np.float32) * np.float32(0.02))
    ids = rng.integers(0, vt, rows).astype(np.int32)
    lg_s = W.logits(c, rows=rows)
    lg_a = W.normal(c, 10, (rows, c.vocab), std=c.logit_std)

    def run():
        O.embedding(ids, table, impl, cores)
        O.residual_rms_norm(x, res, gam, c.eps, impl, cores)
        O.rope(q, k, li["pos"], c.theta, impl, cores)
        O.swiglu(gate, up, impl, cores)
        O.softmax(lg_s, None, impl, cores)
        O.argmax(lg_a, impl, cores)

    return run, sum(step_bytes(rows, 2).values()), kind, cores


def cpu_baseline(seconds=12.0, rows=256, sample=None):
    """Reported CPU baseline: repeat the sample for about `seconds`."""
    run, nbytes, kind, cores = (sample or cpu_sample)(rows)
    run()  # warm-up: page faults, thread start-up
    reps, t0 = 0, time.perf_counter()
    while True:
        run()
        reps += 1
        el = time.perf_counter() - t0
        if el >= seconds or reps >= 500:
            break
    return {"value": round(nbytes * reps / el / 1e9, 3), "unit": "GB/s", "cores": cores,
            "kind": kind,
            "sample": f"{rows} of {CFG.rows} rows of every op of the step, x{reps} "
                      f"({el:.1f} s on {cores} threads)",
            "rows_per_s": round(rows * reps / el, 1)}


def run_reference(args, world):
    """--impl reference: the reference's CPU kernels on this host's cores.
    Each step is one pass of the step's ops over a 256-row sample."""
    rows = 256
    run, nbytes, kind, cores = (cpu_sample_decode(rows) if CFG is CONFIGS["decode"][0]
                                else cpu_sample(rows))
    for _ in range(args.warmup):
        run()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        run()
        times.append(time.perf_counter() - t0)
    sec = statistics.median(times)
    v = round(nbytes / sec / 1e9, 3)
    return {"metric": METRIC, "value": v, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(sec * 1e3, 3), "higher_is_better": True,
            "scaling": "strong" if args.config == "70b" else "weak", "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded, reference config distributions)", "impl": "reference",
            "config": {"workload": WORKLOAD, "rows_sampled": rows, "rows_per_step": CFG.rows},
            "rows_per_s": round(rows / sec, 1),
            "cpu_baseline": {"value": v, "unit": "GB/s", "cores": cores, "kind": kind,
                             "sample": f"{rows} of {CFG.rows} rows of every op per step, "
                                       f"median of {args.steps} steps on {cores} threads"},
            "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


# ------------------------------------------------------------ decode config
def decode_layer_bytes(rows, act_s):
    c = CFG
    return (W.bytes_res_rms(rows, c.hidden, act_s)
            + W.bytes_rope(rows, c.n_q_heads, c.n_kv_heads, c.head_dim, act_s)
            + W.bytes_swiglu(rows, c.intermediate, act_s))


def cpu_sample_decode(rows=256):
    """The decode step on the host cores through the reference's kernels:
    the chain's ops over the batch for DECODE_LAYERS layers, each with its
    own copy of the inputs.  Returns (run, bytes, kind, cores)."""
    import numpy as np
    from oracle import oracle as O
    O.lib()
    impl, kind = (O.REF, "reference") if O.ref_available() else (O.PORT, "port")
    cores = os.cpu_count() or 1
    c = CFG
    li = W.layer_inputs(c, rows=rows)
    bf = O.f32_to_bf16
    one = {k: bf(li[k]) for k in ("x", "res", "gamma", "q", "k", "gate", "up")}
    layers = [{k: np.copy(v) for k, v in one.items()} for _ in range(DECODE_LAYERS)]
    pos = li["pos"]

    def run():
        for d in layers:
            O.residual_rms_norm(d["x"], d["res"], d["gamma"], c.eps, impl, cores)
            O.rope(d["q"], d["k"], pos, c.theta, impl, cores)
            O.swiglu(d["gate"], d["up"], impl, cores)

    return run, DECODE_LAYERS * decode_layer_bytes(rows, 2), kind, cores


def run_decode(args, rank, world, local):
    """One decode step = the fused layer chain over DECODE_LAYERS layers of
    the batch, each layer with its own buffers (1.08 GB per step, so nothing
    is served from L2), captured once in a CUDA graph and replayed."""
    import torch
    import torch.distributed as dist
    import tb_b200 as T

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    L = T.lib()
    R, c, NL = args.rows, CFG, DECODE_LAYERS
    g = torch.Generator(device=dev)

    def randn(shape, seed, std=1.0, mean=0.0):
        g.manual_seed(seed)
        return (torch.randn(shape, generator=g, device=dev) * std + mean).to(torch.bfloat16)

    base = 54321 + 1000 * rank
    g.manual_seed(base)
    pos = torch.randint(0, 4096, (R,), generator=g, device=dev, dtype=torch.int32)
    table = T.rope_table(c.theta, c.head_dim, 4096)
    layers = []
    for l in range(NL):
        sd = base + 16 * l
        d = {"x": randn((R, c.hidden), sd), "res": randn((R, c.hidden), sd + 1),
             "gamma": randn((c.hidden,), sd + 2, 0.1, 1.0),
             "q": randn((R, c.n_q_heads, c.head_dim), sd + 3),
             "k": randn((R, c.n_kv_heads, c.head_dim), sd + 4),
             "gate": randn((R, c.intermediate), sd + 5), "up": randn((R, c.intermediate), sd + 6)}
        d["h"], d["y"], d["act"] = (torch.empty_like(d["x"]), torch.empty_like(d["x"]),
                                    torch.empty_like(d["gate"]))
        d["chain"] = T.make_chain(d["x"], d["res"], d["gamma"], d["h"], d["y"], c.eps, d["q"],
                                  d["k"], pos, c.theta, table, d["gate"], d["up"], d["act"])
        layers.append(d)
    s = torch.cuda.Stream(device=dev)
    sp = C.c_void_p(s.cuda_stream)

    def eager(stream_ptr=sp):
        for d in layers:
            T.check(L.tb_b200_layer_chain(C.byref(d["chain"]), stream_ptr), "layer_chain")

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v):
        if world == 1:
            return v
        x = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(x, op=dist.ReduceOp.MAX)
        return float(x.item())

    s.wait_stream(torch.cuda.current_stream())
    eager()
    s.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        eager()
    with torch.cuda.stream(s):
        for _ in range(args.warmup):
            graph.replay()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    uuid = getattr(torch.cuda.get_device_properties(dev), "uuid", None)
    uuid = f"GPU-{uuid}" if uuid is not None else None
    with ClockSampler(local, uuid) as clocks:
        with torch.cuda.stream(s):
            e0.record(s)
            for _ in range(args.steps):
                graph.replay()
            e1.record(s)
        e1.synchronize()
    torch.cuda.synchronize()
    barrier()
    ms = max_over_ranks(e0.elapsed_time(e1)) / args.steps

    # the same 32 launches without the graph, for the launch overhead
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ke = max(3, min(args.steps, 20))
    a.record(s)
    for _ in range(ke):
        eager()
    b.record(s)
    b.synchronize()
    eager_ms = max_over_ranks(a.elapsed_time(b)) / ke

    # end to end: every layer's inputs copied in and outputs copied out each
    # step, the layers spread over streams so copies overlap the kernels
    ins, outs = ["x", "res", "q", "k", "gate", "up"], ["h", "y", "q", "k", "act"]
    host = [{n: torch.empty_like(d[n], device="cpu").pin_memory() for n in set(ins) | set(outs)}
            for d in layers]
    for d, hd in zip(layers, host):
        for n in ins:
            hd[n].copy_(d[n])
    bi = sum(host[0][n].numel() * host[0][n].element_size() for n in ins) * NL
    bo = sum(host[0][n].numel() * host[0][n].element_size() for n in outs) * NL
    streams = [torch.cuda.Stream(device=dev) for _ in range(E2E_STREAMS)]

    def e2e_step():
        main = torch.cuda.current_stream()
        for st in streams:
            st.wait_stream(main)
        for l, (d, hd) in enumerate(zip(layers, host)):
            ss = C.c_void_p(streams[l % len(streams)].cuda_stream)
            for n in ins:
                T.check(L.tb_b200_memcpy_h2d(T.ptr(d[n]), C.c_void_p(hd[n].data_ptr()),
                                             hd[n].numel() * hd[n].element_size(), ss), "h2d")
            T.check(L.tb_b200_layer_chain(C.byref(d["chain"]), ss), "layer_chain")
            for n in outs:
                T.check(L.tb_b200_memcpy_d2h(C.c_void_p(hd[n].data_ptr()), T.ptr(d[n]),
                                             hd[n].numel() * hd[n].element_size(), ss), "d2h")
        for st in streams:
            main.wait_stream(st)

    stream = torch.cuda.current_stream()
    e2e_step()
    torch.cuda.synchronize()
    barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n2 = max(3, min(args.steps, 10))
    a.record(stream)
    for _ in range(n2):
        e2e_step()
    b.record(stream)
    b.synchronize()
    e2e_ms = max_over_ranks(a.elapsed_time(b)) / n2

    lb = decode_layer_bytes(R, 2)
    step_b = NL * lb
    peak, peak_kind = peaks()
    per_launch = ms / NL
    achieved = lb / (per_launch / 1e3) / 1e9
    total = step_b * world
    return {
        "metric": METRIC, "value": round(total / (ms / 1e3) / 1e9, 1), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded, reference config distributions)",
        "config": {"workload": WORKLOAD, "rows_per_gpu": R, "layers": NL, "hidden": c.hidden,
                   "heads": [c.n_q_heads, c.n_kv_heads, c.head_dim],
                   "intermediate": c.intermediate, "positions": "uniform [0, 4096)",
                   "activations": "bf16 (f32 arithmetic)", "bytes_per_step_per_gpu": step_b,
                   "l2": f"inputs larger than L2: {step_b / 1e9:.2f} GB of distinct per-layer "
                         "buffers per step",
                   "parallelism": f"row-sharded x{world}, no data-path collective"},
        "rows_per_s": round(R * world / (ms / 1e3), 1),
        "per_op": {"layer_chain": {"ms": round(per_launch, 5),
                                   "GB/s": round(lb / per_launch / 1e6, 1),
                                   "frac": round(lb / per_launch / 1e6 / peak, 3), "bytes": lb}},
        "eager_ms_per_step": round(eager_ms, 4),
        "roofline": {"bound": "hbm", "kernel": "layer_chain", "achieved": round(achieved, 1),
                     "peak": peak, "peak_source": peak_kind, "unit": "GB/s",
                     "frac": round(achieved / peak, 3),
                     "traffic": round(TRAFFIC_PER_ROW["7b"]["layer_chain"] * R),
                     "algorithmic_bytes": lb,
                     "traffic_source": TRAFFIC_SOURCE + "; captured at the same row shape",
                     "duration": "graph step time / layers (launch gaps included)"},
        "e2e": {"value": round(total / (e2e_ms / 1e3) / 1e9, 2), "unit": "GB/s",
                "ms_per_step": round(e2e_ms, 3), "h2d_bytes_per_step": bi,
                "d2h_bytes_per_step": bo,
                "api": f"tb_b200_* C ABI, pinned host buffers, layers on {len(streams)} streams"},
        "gpu_launches": NL * args.steps,
        "clocks": clocks.summary(),
    }


# ------------------------------------------------------------ runner config
PATTERNS_2_4 = (0x3, 0x5, 0x6, 0x9, 0xA, 0xC)


def runner_cfg(layers):
    c = CFG
    return dict(hidden=c.hidden, n_heads=c.n_q_heads, n_kv_heads=c.n_kv_heads,
                head_dim=c.head_dim, intermediate=c.intermediate, vocab=c.vocab,
                max_seq=RUNNER_MAX_SEQ, layers=layers, norm_eps=c.eps, rope_theta=c.theta)


def runner_shapes(cfg):
    H, I = cfg["hidden"], cfg["intermediate"]
    qd, kvd = cfg["n_heads"] * cfg["head_dim"], cfg["n_kv_heads"] * cfg["head_dim"]
    return dict(q=(qd, H), k=(kvd, H), v=(kvd, H), o=(H, qd), gate=(I, H), up=(I, H),
                down=(H, I))


def runner_token_bytes(cfg, pos, int4=False):
    """Algorithmic bytes of one token at position `pos` in the runner's
    layout: packed 2:4 projections (kept f32 values + index bytes) or INT4
    projections (bytes + scales), the dense f32 lm head, the embedding row,
    the norm weights, and the KV cache (rows 0..pos-1 read for every layer,
    row pos written)."""
    H, L = cfg["hidden"], cfg["layers"]
    kvd = cfg["n_kv_heads"] * cfg["head_dim"]
    proj = 0
    for rows, cols in runner_shapes(cfg).values():
        if int4:  # half a byte per weight, a 4-byte scale per group
            proj += rows * cols // 2 + rows * cols // RUNNER_GROUP * 4
            continue
        pairs = cols // 8
        proj += rows * pairs * 16 + rows * ((pairs + 127) // 128 * 128)
    return (L * proj + cfg["vocab"] * H * 4 + H * 4 + (2 * L + 1) * H * 4
            + L * 2 * kvd * 4 * (pos + 1))


def runner_model_torch(torch, dev, cfg, seed, int4=False):
    """Weights U(-0.01, 0.01) (the engine's mock initialisation), random 2:4
    masks, norm weights 1 + N(0, 0.1); all f32 on the device.  int4: the
    projections are random INT4 bytes with scales per 128 weights."""
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    pats = torch.tensor(PATTERNS_2_4, dtype=torch.uint8, device=dev)

    def w(r, c):
        return (torch.rand((r, c), generator=g, device=dev) - 0.5) * 0.02

    def nv():
        return 1 + 0.1 * torch.randn(cfg["hidden"], generator=g, device=dev)

    def q4(r, c):  # random INT4 bytes, scales U(0, 0.002)
        import tb_b200 as T
        data = torch.randint(0, 256, (r * c // 2,), dtype=torch.uint8, generator=g, device=dev)
        scales = torch.rand(r * c // RUNNER_GROUP, generator=g, device=dev) * 0.002
        return (T.QuantWeight(data, T.INT4, r, c, scales, RUNNER_GROUP), None)

    layers = []
    for _ in range(cfg["layers"]):
        if int4:
            ly = {n: q4(r, c) for n, (r, c) in runner_shapes(cfg).items()}
        else:
            ly = {n: (w(r, c), pats[torch.randint(0, len(PATTERNS_2_4), (r, c // 4), generator=g,
                                                  device=dev)].contiguous())
                  for n, (r, c) in runner_shapes(cfg).items()}
        ly["in_norm"], ly["post_norm"] = nv(), nv()
        layers.append(ly)
    return dict(embed=w(cfg["vocab"], cfg["hidden"]), final_norm=nv(),
                lm_head=w(cfg["vocab"], cfg["hidden"]), layers=layers)


def cpu_sample_runner(seconds=10.0):
    """The reference runner's arithmetic on the host (the oracle's
    restatement, oracle/runner.c; the reference's own runner reads past its
    norm weights at this shape, vocab > hidden): one token through models
    of 0 and 2 layers of the llama7b shape, scaled to 32 layers.  The
    sample token is at position 0: the host's attention over a 1024-token
    context is left out, so the baseline is, if anything, fast."""
    import numpy as np
    from oracle import oracle as O
    rng = np.random.default_rng(7)
    pats = np.array(PATTERNS_2_4, np.uint8)

    def model(layers):
        cfg = runner_cfg(layers)
        lys = []
        for _ in range(layers):
            ly = {n: (((rng.random((r, c), dtype=np.float32) - 0.5) * 0.02),
                      pats[rng.integers(0, 6, (r, c // 4))])
                  for n, (r, c) in runner_shapes(cfg).items()}
            ly["in_norm"] = ly["post_norm"] = np.ones(cfg["hidden"], np.float32)
            lys.append(ly)
        emb = ((rng.random((cfg["vocab"], cfg["hidden"]), dtype=np.float32) - 0.5) * 0.02)
        return cfg, dict(embed=emb, final_norm=None, lm_head=None, layers=lys)

    def timed(cfg, m):
        O.runner_run(cfg, m, np.array([1], np.int32))  # warm-up
        reps, t0 = 0, time.perf_counter()
        while True:
            O.runner_run(cfg, m, np.array([1], np.int32))
            reps += 1
            if time.perf_counter() - t0 >= seconds / 2 or reps >= 20:
                break
        return (time.perf_counter() - t0) / reps

    t0 = timed(*model(0))
    t2 = timed(*model(2))
    per_token = t0 + RUNNER_LAYERS * max(t2 - t0, 0.0) / 2
    return per_token, ("one token through 0- and 2-layer llama7b-shape models (oracle/runner.c, "
                       "1 thread), scaled to 32 layers")


def run_runner(args, rank, world, local):
    """One step = one token of a single sequence through the device runner
    (tb_b200_runner_forward, a CUDA graph) after a context of RUNNER_CONTEXT
    tokens, so every timed token attends over 1024+ cached positions; every
    rank runs its own replica (no exchange on this path)."""
    import torch
    import torch.distributed as dist
    import tb_b200 as T

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    cfg = runner_cfg(args.runner_layers)
    int4 = args.config == "runner_int4"
    model = runner_model_torch(torch, dev, cfg, 777 + rank, int4=int4)
    runner = T.Runner(cfg, model, attention=T.ATTN_STANDARD, use_graph=True)
    stream = torch.cuda.ExternalStream(runner.stream.value)
    n_tok = RUNNER_CONTEXT + args.warmup + args.steps + max(3, min(args.steps, 20)) + 8
    if n_tok > RUNNER_MAX_SEQ:
        raise SystemExit(f"--config runner: {n_tok} positions exceed max_seq {RUNNER_MAX_SEQ}")
    tokens = torch.randint(0, cfg["vocab"], (n_tok,),
                           generator=torch.Generator().manual_seed(5)).tolist()

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    it = iter(tokens)
    for _ in range(RUNNER_CONTEXT + args.warmup):  # the context, then the warm-up tokens
        runner.forward(next(it))
    torch.cuda.synchronize()
    pos0 = runner.position
    uuid = getattr(torch.cuda.get_device_properties(dev), "uuid", None)
    uuid = f"GPU-{uuid}" if uuid is not None else None
    barrier()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local, uuid) as clocks:
        a.record(stream)
        for _ in range(args.steps):
            runner.forward(next(it))
        b.record(stream)
        b.synchronize()
    ms = max_over_ranks(a.elapsed_time(b)) / args.steps
    launches = runner.launches_per_token * args.steps

    # end to end: the token id in from the host, the logits out to it, every token
    barrier()
    torch.cuda.synchronize()
    n2 = max(3, min(args.steps, 20))
    a.record(stream)
    for _ in range(n2):
        runner.forward(next(it))
        runner.logits()
    b.record(stream)
    b.synchronize()
    e2e_ms = max_over_ranks(a.elapsed_time(b)) / n2
    runner.close()

    mean_pos = pos0 + (args.steps - 1) / 2
    tb = runner_token_bytes(cfg, mean_pos, int4=int4)
    peak, peak_kind = peaks()
    achieved = tb / (ms / 1e3) / 1e9
    tok_s = world * 1e3 / ms
    return {
        "metric": RUNNER_METRIC, "value": round(tok_s, 2), "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int4 weights, f32 arithmetic" if int4 else "f32",
        "data": ("synthetic (seeded; random INT4 projections, scales per 128 weights, "
                 "norm weights 1 + N(0, 0.1))" if int4 else
                 "synthetic (seeded; weights U(-0.01, 0.01) as the engine's mock model, "
                 "random 2:4 masks, norm weights 1 + N(0, 0.1))"),
        "config": {"workload": WORKLOAD, "layers": cfg["layers"], "hidden": cfg["hidden"],
                   "heads": [cfg["n_heads"], cfg["n_kv_heads"], cfg["head_dim"]],
                   "intermediate": cfg["intermediate"], "vocab": cfg["vocab"],
                   "max_seq": RUNNER_MAX_SEQ, "attention": "standard (every key of the row)",
                   "context": f"{RUNNER_CONTEXT} tokens fed untimed before the warm-up",
                   "positions": f"{pos0} .. {pos0 + args.steps - 1}",
                   "bytes_per_token_per_gpu": tb,
                   "l2": f"inputs larger than L2: {tb / 1e9:.1f} GB of weights per token",
                   "parallelism": f"replicas x{world}, no data-path collective"},
        "roofline": {"bound": "hbm", "kernel": "decoder step (every kernel of a token)",
                     "achieved": round(achieved, 1), "peak": peak, "peak_source": peak_kind,
                     "unit": "GB/s", "frac": round(achieved / peak, 3), "traffic": None,
                     "algorithmic_bytes": tb,
                     "traffic_source": "no ncu capture of the whole step",
                     "duration": "graph replay time per token"},
        "e2e": {"value": round(world * 1e3 / e2e_ms, 2), "unit": "tokens/s",
                "ms_per_step": round(e2e_ms, 3), "h2d_bytes_per_step": 4,
                "d2h_bytes_per_step": cfg["vocab"] * 4,
                "api": "tb_b200_runner_forward + tb_b200_runner_logits (token id in, logits "
                       "out, synchronous per token)"},
        "gpu_launches": int(launches),
        "clocks": clocks.summary(),
    }


def run_reference_runner(args, world):
    per_token, sample = cpu_sample_runner()
    v = round(1.0 / per_token, 4)
    return {"metric": RUNNER_METRIC, "value": v, "unit": "tokens/s", "n_gpus": world,
            "steps": 1, "warmup": 1, "ms_per_step": round(per_token * 1e3, 1),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded)", "impl": "reference",
            "config": {"workload": WORKLOAD, "layers": RUNNER_LAYERS},
            "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": 1, "kind": "port",
                             "sample": sample},
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


# ------------------------------------------------------------------ GPU arm
def build_inputs(torch, dev, seed, rows=None):
    c = CFG
    g = torch.Generator(device=dev)

    def randn(shape, std=1.0, mean=0.0, dtype=torch.bfloat16, k=0):
        g.manual_seed(seed + k)
        return (torch.randn(shape, generator=g, device=dev) * std + mean).to(dtype)

    R = c.rows if rows is None else rows
    LR = logit_rows(R)
    t = {
        "table": randn((c.vocab, c.hidden), 0.02, k=7),
        "ids": torch.randint(0, c.vocab, (R,), generator=g, device=dev, dtype=torch.int32),
        "x": randn((R, c.hidden), k=0), "res": randn((R, c.hidden), k=1),
        "gamma": randn((c.hidden,), 0.1, 1.0, k=2),
        "q": randn((R, c.n_q_heads, c.head_dim), k=3), "k": randn((R, c.n_kv_heads, c.head_dim), k=4),
        "gate": randn((R, c.intermediate), k=5), "up": randn((R, c.intermediate), k=6),
        "pos": torch.arange(R, dtype=torch.int32, device=dev),
        "logits_s": randn((LR, c.vocab), c.logit_std, dtype=torch.float32, k=9),
        "logits_a": randn((LR, c.vocab), c.logit_std, dtype=torch.float32, k=10),
    }
    o = {
        "emb": torch.empty((R, c.hidden), dtype=torch.bfloat16, device=dev),
        "h": torch.empty_like(t["x"]), "y": torch.empty_like(t["x"]),
        "act": torch.empty_like(t["gate"]),
        "probs": torch.empty_like(t["logits_s"]),
        "tok": torch.empty(LR, dtype=torch.int32, device=dev),
    }
    return t, o


def run_gpu(args, rank, world, local):
    import torch
    import torch.distributed as dist
    import tb_b200 as T

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    L = T.lib()
    R, c = args.rows, CFG
    LR = logit_rows(R)
    t, o = build_inputs(torch, dev, 12345 + 1000 * rank, R)
    table = T.rope_table(CFG.theta, CFG.head_dim, R)
    stream = torch.cuda.current_stream()
    sp = C.c_void_p(stream.cuda_stream)
    chain = T.make_chain(t["x"], t["res"], t["gamma"], o["h"], o["y"], CFG.eps, t["q"], t["k"],
                         t["pos"], CFG.theta, table, t["gate"], t["up"], o["act"])

    ops = {
        "embedding": lambda: T.check(L.tb_b200_embedding(T.BF16, R, c.hidden, c.vocab, T.ptr(t["ids"]),
                                                         T.ptr(t["table"]), T.ptr(o["emb"]), sp),
                                     "embedding"),
        "layer_chain": lambda: T.check(L.tb_b200_layer_chain(C.byref(chain), sp), "layer_chain"),
        "softmax": lambda: T.check(L.tb_b200_softmax(T.F32, LR, c.vocab, T.ptr(t["logits_s"]), None,
                                                     T.ptr(o["probs"]), sp), "softmax"),
        "argmax": lambda: T.check(L.tb_b200_argmax(T.F32, LR, c.vocab, T.ptr(t["logits_a"]),
                                                   T.ptr(o["tok"]), sp), "argmax"),
    }

    def step():
        for f in ops.values():
            f()

    if args.profile_op:
        for _ in range(args.warmup + args.steps):
            ops[args.profile_op]()
        torch.cuda.synchronize()
        return None

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v):
        if world == 1:
            return v
        x = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(x, op=dist.ReduceOp.MAX)
        return float(x.item())

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    l0 = L.tb_b200_launch_count()
    uuid = getattr(torch.cuda.get_device_properties(dev), "uuid", None)
    uuid = f"GPU-{uuid}" if uuid is not None else None
    with ClockSampler(local, uuid) as clocks:
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        e1.synchronize()
    launches = L.tb_b200_launch_count() - l0
    torch.cuda.synchronize()
    barrier()
    ms_total = max_over_ranks(e0.elapsed_time(e1))
    ms = ms_total / args.steps

    # per-kernel device time inside full steps (for the roofline)
    names = list(ops)
    evs = {n: [] for n in names}
    for _ in range(max(3, min(args.steps, 50))):
        for n in names:
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            ops[n]()
            b.record(stream)
            evs[n].append((a, b))
    torch.cuda.synchronize()
    per_op_ms = {n: statistics.mean(a.elapsed_time(b) for a, b in evs[n]) for n in names}
    parts = step_bytes(R, 2)
    step_b = sum(parts.values())
    peak, peak_kind = peaks()
    dom = max(per_op_ms, key=per_op_ms.get)
    achieved = parts[dom] / (per_op_ms[dom] / 1e3) / 1e9
    per_op = {n: {"ms": round(per_op_ms[n], 4), "GB/s": round(parts[n] / per_op_ms[n] / 1e6, 1),
                  "frac": round(parts[n] / per_op_ms[n] / 1e6 / peak, 3),
                  "bytes": parts[n]} for n in names}

    # End to end through the C ABI: pinned host inputs in, outputs back out,
    # every step.  The rows are independent, so the step runs as E2E_BLOCKS
    # row blocks spread over E2E_STREAMS streams, each block copying its own
    # inputs in, running the four ops on its rows and copying its outputs
    # out: one block's host-to-device copy overlaps the others' kernels and
    # device-to-host copies (separate copy engines).  Weights (embedding
    # table, RMSNorm gamma, RoPE table) stay resident.
    ins = ["ids", "x", "res", "q", "k", "gate", "up", "logits_s", "logits_a"]
    outs = ["emb", "h", "y", "q", "k", "act", "probs", "tok"]
    host_in = {n: torch.empty_like(t[n], device="cpu").pin_memory() for n in ins}
    for n in ins:
        host_in[n].copy_(t[n])
    host_out = {n: torch.empty_like((o.get(n) if n in o else t[n]), device="cpu").pin_memory()
                for n in outs}
    bi = sum(host_in[n].numel() * host_in[n].element_size() for n in ins)
    bo = sum(host_out[n].numel() * host_out[n].element_size() for n in outs)
    nb = E2E_BLOCKS if R % E2E_BLOCKS == 0 and LR % E2E_BLOCKS == 0 else 1
    rb, lrb = R // nb, LR // nb
    logit_names = {"logits_s", "logits_a", "probs", "tok"}  # LR rows, the rest R
    streams = [torch.cuda.Stream(device=dev) for _ in range(E2E_STREAMS)]

    def dev_of(n):
        return o[n] if n in o else t[n]

    blocks = []
    for j in range(nb):
        span = {n: ((j * lrb, (j + 1) * lrb) if n in logit_names else (j * rb, (j + 1) * rb))
                for n in set(ins) | set(outs)}
        sl = {n: dev_of(n)[a:b] for n, (a, b) in span.items()}
        sl["pos"] = t["pos"][j * rb:(j + 1) * rb]
        ch = T.make_chain(sl["x"], sl["res"], t["gamma"], sl["h"], sl["y"], CFG.eps, sl["q"],
                          sl["k"], sl["pos"], CFG.theta, table, sl["gate"], sl["up"], sl["act"])
        blocks.append((span, sl, ch))

    def e2e_step():
        main = torch.cuda.current_stream()
        for st in streams:
            st.wait_stream(main)
        for j, (span, sl, ch) in enumerate(blocks):
            st = streams[j % len(streams)]
            ss = C.c_void_p(st.cuda_stream)
            for n in ins:
                hb = host_in[n][span[n][0]:span[n][1]]
                T.check(L.tb_b200_memcpy_h2d(T.ptr(sl[n]), C.c_void_p(hb.data_ptr()),
                                             hb.numel() * hb.element_size(), ss), "h2d")
            T.check(L.tb_b200_embedding(T.BF16, rb, c.hidden, c.vocab, T.ptr(sl["ids"]),
                                        T.ptr(t["table"]), T.ptr(sl["emb"]), ss), "embedding")
            T.check(L.tb_b200_layer_chain(C.byref(ch), ss), "layer_chain")
            T.check(L.tb_b200_softmax(T.F32, lrb, c.vocab, T.ptr(sl["logits_s"]), None,
                                      T.ptr(sl["probs"]), ss), "softmax")
            T.check(L.tb_b200_argmax(T.F32, lrb, c.vocab, T.ptr(sl["logits_a"]),
                                     T.ptr(sl["tok"]), ss), "argmax")
            for n in outs:
                hb = host_out[n][span[n][0]:span[n][1]]
                T.check(L.tb_b200_memcpy_d2h(C.c_void_p(hb.data_ptr()), T.ptr(sl[n]),
                                             hb.numel() * hb.element_size(), ss), "d2h")
        for st in streams:
            main.wait_stream(st)

    e2e_steps = max(3, min(args.steps, 10))
    e2e_step()
    torch.cuda.synchronize()
    barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    b.record(stream)
    b.synchronize()
    e2e_ms = max_over_ranks(a.elapsed_time(b)) / e2e_steps

    total_bytes = step_b * world
    line = {
        "metric": METRIC, "value": round(total_bytes / (ms / 1e3) / 1e9, 1), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded, reference config distributions)",
        "config": {"workload": WORKLOAD, "rows_per_gpu": R, "hidden": c.hidden,
                   "heads": [c.n_q_heads, c.n_kv_heads, c.head_dim],
                   "intermediate": c.intermediate, "vocab": c.vocab,
                   "activations": "bf16 (f32 arithmetic)", "logits": "f32",
                   "logit_rows_per_gpu": LR, "bytes_per_step_per_gpu": step_b,
                   "l2": f"inputs larger than L2: {step_b / 1e9:.1f} GB of distinct buffers per step",
                   "parallelism": f"row-sharded x{world}, no data-path collective"},
        "rows_per_s": round(R * world / (ms / 1e3), 1),
        "per_op": per_op,
        "roofline": {"bound": "hbm", "kernel": dom, "achieved": round(achieved, 1),
                     "peak": peak, "peak_source": peak_kind, "unit": "GB/s",
                     "frac": round(achieved / peak, 3),
                     "traffic": (round(TRAFFIC_PER_ROW["7b"][dom] * (LR if dom in ("softmax", "argmax") else R))
                                 if CFG is CONFIGS["7b"][0] else None),
                     "algorithmic_bytes": parts[dom],
                     "traffic_source": (TRAFFIC_SOURCE if CFG is CONFIGS["7b"][0] else
                                        "no ncu capture of this configuration")},
        "e2e": {"value": round(total_bytes / (e2e_ms / 1e3) / 1e9, 2), "unit": "GB/s",
                "ms_per_step": round(e2e_ms, 3), "h2d_bytes_per_step": bi,
                "d2h_bytes_per_step": bo,
                "api": f"tb_b200_* C ABI, pinned host buffers, {nb} row blocks on "
                       f"{len(streams)} streams (copies in and out overlap the kernels)"},
        "gpu_launches": int(launches),
        "clocks": clocks.summary(),
    }
    return line


# ----------------------------------------------- 70b prefill, strong-scaled
def table_shard(torch, dev, c, lo, hi, seed):
    """Rows [lo, hi) of the [vocab, hidden] bf16 embedding table ~N(0, 0.02).
    The table is drawn TABLE_CHUNK rows at a time, chunk j from seed + j, so
    a rank's shard is a slice of the same table whatever the rank count."""
    out = torch.empty((hi - lo, c.hidden), dtype=torch.bfloat16, device=dev)
    g = torch.Generator(device=dev)
    if hi <= lo:
        return out
    for j in range(lo // TABLE_CHUNK, (hi - 1) // TABLE_CHUNK + 1):
        a, b = j * TABLE_CHUNK, min((j + 1) * TABLE_CHUNK, c.vocab)
        g.manual_seed(seed + j)
        blk = (torch.randn((b - a, c.hidden), generator=g, device=dev) * 0.02).to(torch.bfloat16)
        lo2, hi2 = max(a, lo), min(b, hi)
        out[lo2 - lo:hi2 - lo] = blk[lo2 - a:hi2 - a]
    return out


def run_sharded(args, rank, world, local):
    """The 70b step strong-scaled over `world` ranks: rank r takes token
    rows tb_b200_partition(16384, world, r), logit rows
    tb_b200_partition(4096, world, r) and table rows
    tb_b200_partition(128256, world, r).  The embedding gather is the
    library's one-kernel gather over its communicator's symmetric memory
    (NCCL windows; the NCCL send/recv exchange and the CUDA IPC gather are
    timed beside it); every other op is local to the rank."""
    import numpy as np
    import torch
    import torch.distributed as dist
    import tb_b200 as T

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    L = T.lib()
    c = CFG
    NT, NLG = args.rows, LOGIT_ROWS
    tlo, thi = T.partition(NT, world, rank)
    llo, lhi = T.partition(NLG, world, rank)
    vlo, vhi = T.partition(c.vocab, world, rank)
    R, LR = thi - tlo, lhi - llo

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v, op=None):
        if world == 1:
            return v
        x = torch.tensor([float(v)], dtype=torch.float64, device=dev)
        dist.all_reduce(x, op=op or dist.ReduceOp.MAX)
        return float(x.item())

    if args.profile_op in ("softmax", "argmax"):
        # a small case for ncu: only this op's buffers (world 1)
        g = torch.Generator(device=dev)
        g.manual_seed(12345 + 9)
        x = torch.empty((LR, c.vocab), device=dev).normal_(0.0, c.logit_std, generator=g)
        out = (torch.empty_like(x) if args.profile_op == "softmax"
               else torch.empty(LR, dtype=torch.int32, device=dev))
        sp = C.c_void_p(torch.cuda.current_stream().cuda_stream)
        for _ in range(args.warmup + args.steps):
            if args.profile_op == "softmax":
                T.check(L.tb_b200_softmax(T.F32, LR, c.vocab, T.ptr(x), None, T.ptr(out), sp),
                        "softmax")
            else:
                T.check(L.tb_b200_argmax(T.F32, LR, c.vocab, T.ptr(x), T.ptr(out), sp), "argmax")
        torch.cuda.synchronize()
        return None

    # the library's NCCL communicator over the same ranks
    if world > 1:
        uid = [T.comm_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        uid = uid[0]
    else:
        uid = T.comm_unique_id()
    T.comm_init(world, rank, uid, local)

    ids = np.random.default_rng(c.seed + 8).integers(0, c.vocab, NT).astype(np.int32)
    table_seed = c.seed + 700
    shard = table_shard(torch, dev, c, vlo, vhi, table_seed)
    # The table part in the communicator's symmetric memory: every rank's
    # window has the size of the largest part.
    win_bytes = -(-c.vocab // world) * c.hidden * 2
    win = T.comm_window_alloc(win_bytes)
    T.check(L.tb_b200_memcpy_d2d(C.c_void_p(win), T.ptr(shard), shard.numel() * 2, None), "d2d")
    torch.cuda.synchronize()
    barrier()  # every part written before any rank gathers
    my_ids = torch.from_numpy(ids[tlo:thi]).to(dev)
    g = torch.Generator(device=dev)
    base = 12345 + 1000 * rank

    def randn(shape, std=1.0, mean=0.0, dtype=torch.bfloat16, k=0):
        g.manual_seed(base + k)
        return (torch.randn(shape, generator=g, device=dev) * std + mean).to(dtype)

    t = {
        "x": randn((R, c.hidden), k=0), "res": randn((R, c.hidden), k=1),
        "gamma": randn((c.hidden,), 0.1, 1.0, k=2),
        "q": randn((R, c.n_q_heads, c.head_dim), k=3),
        "k": randn((R, c.n_kv_heads, c.head_dim), k=4),
        "gate": randn((R, c.intermediate), k=5), "up": randn((R, c.intermediate), k=6),
        "pos": (torch.arange(tlo, thi, dtype=torch.int32, device=dev) % SEQ_LEN_70B),
        "logits_s": randn((LR, c.vocab), c.logit_std, dtype=torch.float32, k=9),
        "logits_a": randn((LR, c.vocab), c.logit_std, dtype=torch.float32, k=10),
    }
    o = {
        "emb": torch.empty((R, c.hidden), dtype=torch.bfloat16, device=dev),
        "h": torch.empty_like(t["x"]), "y": torch.empty_like(t["x"]),
        "act": torch.empty_like(t["gate"]), "probs": torch.empty_like(t["logits_s"]),
        "tok": torch.empty(LR, dtype=torch.int32, device=dev),
    }
    rope = T.rope_table(c.theta, c.head_dim, SEQ_LEN_70B)
    stream = torch.cuda.current_stream()
    sp = C.c_void_p(stream.cuda_stream)
    chain = T.make_chain(t["x"], t["res"], t["gamma"], o["h"], o["y"], c.eps, t["q"], t["k"],
                         t["pos"], c.theta, rope, t["gate"], t["up"], o["act"])
    ids_p = ids.ctypes.data
    ops = {
        "embedding": lambda: T.check(L.tb_b200_embedding_sharded_window(
            T.BF16, R, c.hidden, c.vocab, T.ptr(my_ids), C.c_void_p(win), T.ptr(o["emb"]), sp),
            "embedding_sharded_window"),
        "layer_chain": lambda: T.check(L.tb_b200_layer_chain(C.byref(chain), sp), "layer_chain"),
        "softmax": lambda: T.check(L.tb_b200_softmax(T.F32, LR, c.vocab, T.ptr(t["logits_s"]),
                                                     None, T.ptr(o["probs"]), sp), "softmax"),
        "argmax": lambda: T.check(L.tb_b200_argmax(T.F32, LR, c.vocab, T.ptr(t["logits_a"]),
                                                   T.ptr(o["tok"]), sp), "argmax"),
    }

    def step():
        for f in ops.values():
            f()

    # The same gather two other ways, each timed alone: the NCCL exchange
    # (host ids, a host plan, pack, grouped send/recv, scatter) and one
    # kernel over CUDA IPC mappings of the other ranks' parts.
    if world > 1:
        handles = [None] * world
        dist.all_gather_object(handles, T.p2p_export(shard))
        addrs = [shard.data_ptr() if r == rank else T.p2p_import(*handles[r])
                 for r in range(world)]
    else:
        handles, addrs = None, [shard.data_ptr()]
    y_p2p = torch.empty_like(o["emb"])
    y_nccl = torch.empty_like(o["emb"])
    darr = (C.c_void_p * world)(*addrs)

    def p2p():
        T.check(L.tb_b200_embedding_sharded_p2p(T.BF16, R, c.hidden, c.vocab, T.ptr(my_ids), darr,
                                                world, T.ptr(y_p2p), sp), "embedding_sharded_p2p")

    def nccl():
        T.check(L.tb_b200_embedding_sharded(T.BF16, NT, c.hidden, c.vocab, ids_p, C.c_void_p(win),
                                            T.ptr(y_nccl), sp), "embedding_sharded")

    if args.profile_op:
        f = {"embedding_nccl": nccl, "embedding_ipc": p2p}.get(args.profile_op)
        for _ in range(args.warmup + args.steps):
            (f or ops[args.profile_op])()
        torch.cuda.synchronize()
        barrier()
        T.comm_destroy()
        return None

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    l0 = L.tb_b200_launch_count()
    uuid = getattr(torch.cuda.get_device_properties(dev), "uuid", None)
    uuid = f"GPU-{uuid}" if uuid is not None else None
    with ClockSampler(local, uuid) as clocks:
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        e1.synchronize()
    launches = L.tb_b200_launch_count() - l0
    torch.cuda.synchronize()
    barrier()
    ms = max_over_ranks(e0.elapsed_time(e1)) / args.steps

    # per-op device time inside full steps (for the roofline and the shares)
    names = list(ops)
    evs = {n: [] for n in names}
    for _ in range(max(3, min(args.steps, 20))):
        for n in names:
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            ops[n]()
            b.record(stream)
            evs[n].append((a, b))
    torch.cuda.synchronize()
    per_op_ms = {n: max_over_ranks(statistics.mean(a.elapsed_time(b) for a, b in evs[n]))
                 for n in names}
    barrier()

    def time_alone(f, n):
        for _ in range(3):
            f()
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(n):
            f()
        b.record(stream)
        b.synchronize()
        return max_over_ranks(a.elapsed_time(b)) / n

    n_side = max(5, min(args.steps, 20))
    win_ms = time_alone(ops["embedding"], n_side)
    p2p_ms = time_alone(p2p, n_side)
    nccl_ms = time_alone(nccl, n_side)
    # all three gathers against each other and against the table itself: a
    # sample of token rows regenerated from their chunk's seed
    ops["embedding"]()
    torch.cuda.synchronize()
    as16 = lambda t: t.view(torch.int16)  # noqa: E731
    same = bool(torch.equal(as16(o["emb"]), as16(y_p2p)) and torch.equal(as16(o["emb"]), as16(y_nccl)))
    rs = np.random.default_rng(11 + rank)
    sample = sorted(set(rs.integers(0, R, 8).tolist()) | {0, R - 1}) if R else []
    by_chunk = {}
    for r_ in sample:
        by_chunk.setdefault(int(ids[tlo + r_]) // TABLE_CHUNK, []).append(r_)
    for j, rows_ in by_chunk.items():
        lo_, hi_ = j * TABLE_CHUNK, min((j + 1) * TABLE_CHUNK, c.vocab)
        chunk = table_shard(torch, dev, c, lo_, hi_, table_seed)
        for r_ in rows_:
            same = same and bool(torch.equal(as16(o["emb"][r_]),
                                              as16(chunk[int(ids[tlo + r_]) - lo_])))
        del chunk
    verified = max_over_ranks(0.0 if same else 1.0) == 0.0
    if world > 1:
        torch.cuda.synchronize()
        for r in range(world):
            if r != rank:
                T.p2p_close(addrs[r], handles[r][1])
        barrier()  # every importer closed before an owner may free its shard
    owner = np.searchsorted(np.array([T.partition(c.vocab, world, r)[1] for r in range(world)]),
                            ids[tlo:thi], side="right")
    n_remote = int((owner != rank).sum())
    nvlink_bytes = max_over_ranks(n_remote * c.hidden * 2)

    # End to end through the C ABI: pinned host inputs in, outputs back out,
    # every step.  The gather takes its host ids as the engine passes them;
    # the other ops run as row blocks spread over streams, each block copying
    # its own inputs in and its outputs out, so copies overlap kernels.
    ins = ["x", "res", "q", "k", "gate", "up", "logits_s", "logits_a"]
    outs = ["emb", "h", "y", "q", "k", "act", "probs", "tok"]
    host_in = {n: torch.empty_like(t[n], device="cpu").pin_memory() for n in ins}
    for n in ins:
        host_in[n].copy_(t[n])
    host_out = {n: torch.empty_like((o.get(n) if n in o else t[n]), device="cpu").pin_memory()
                for n in outs}
    bi = sum(host_in[n].numel() * host_in[n].element_size() for n in ins) + 4 * R
    bo = sum(host_out[n].numel() * host_out[n].element_size() for n in outs)
    nb = E2E_BLOCKS if R % E2E_BLOCKS == 0 and LR % E2E_BLOCKS == 0 else 1
    rb, lrb = R // nb, LR // nb
    logit_names = {"logits_s", "logits_a", "probs", "tok"}
    streams = [torch.cuda.Stream(device=dev) for _ in range(E2E_STREAMS)]

    def dev_of(n):
        return o[n] if n in o else t[n]

    blocks = []
    for j in range(nb):
        span = {n: ((j * lrb, (j + 1) * lrb) if n in logit_names else (j * rb, (j + 1) * rb))
                for n in set(ins) | set(outs)}
        sl = {n: dev_of(n)[a_:b_] for n, (a_, b_) in span.items()}
        sl["pos"] = t["pos"][j * rb:(j + 1) * rb]
        ch = T.make_chain(sl["x"], sl["res"], t["gamma"], sl["h"], sl["y"], c.eps, sl["q"],
                          sl["k"], sl["pos"], c.theta, rope, sl["gate"], sl["up"], sl["act"])
        blocks.append((span, sl, ch))

    ids_host = torch.from_numpy(ids[tlo:thi].copy()).pin_memory()

    def e2e_step():
        main = torch.cuda.current_stream()
        for st in streams:
            st.wait_stream(main)
        # this rank's ids in, then the gather, on the main stream
        T.check(L.tb_b200_memcpy_h2d(T.ptr(my_ids), C.c_void_p(ids_host.data_ptr()), R * 4, sp),
                "h2d")
        ops["embedding"]()
        gathered = torch.cuda.Event()
        gathered.record(main)
        for j, (span, sl, ch) in enumerate(blocks):
            st = streams[j % len(streams)]
            ss = C.c_void_p(st.cuda_stream)
            for n in ins:
                hb = host_in[n][span[n][0]:span[n][1]]
                T.check(L.tb_b200_memcpy_h2d(T.ptr(sl[n]), C.c_void_p(hb.data_ptr()),
                                             hb.numel() * hb.element_size(), ss), "h2d")
            T.check(L.tb_b200_layer_chain(C.byref(ch), ss), "layer_chain")
            T.check(L.tb_b200_softmax(T.F32, lrb, c.vocab, T.ptr(sl["logits_s"]), None,
                                      T.ptr(sl["probs"]), ss), "softmax")
            T.check(L.tb_b200_argmax(T.F32, lrb, c.vocab, T.ptr(sl["logits_a"]),
                                     T.ptr(sl["tok"]), ss), "argmax")
            st.wait_event(gathered)
            for n in outs:
                hb = host_out[n][span[n][0]:span[n][1]]
                T.check(L.tb_b200_memcpy_d2h(C.c_void_p(hb.data_ptr()), T.ptr(sl[n]),
                                             hb.numel() * hb.element_size(), ss), "d2h")
        for st in streams:
            main.wait_stream(st)

    e2e_steps = max(3, min(args.steps, 5))
    e2e_step()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    b.record(stream)
    b.synchronize()
    e2e_ms = max_over_ranks(a.elapsed_time(b)) / e2e_steps
    torch.cuda.synchronize()
    barrier()
    T.comm_window_free(win)
    T.comm_destroy()

    parts = step_bytes(NT, 2, NLG)  # the whole job's algorithmic bytes
    total_bytes = sum(parts.values())
    mine = step_bytes(R, 2, LR)    # this rank's share
    peak, peak_kind = peaks()
    dom = max(per_op_ms, key=per_op_ms.get)
    achieved = mine[dom] / (per_op_ms[dom] / 1e3) / 1e9
    step_sum = sum(per_op_ms.values())
    per_op = {n: {"ms": round(per_op_ms[n], 4), "GB/s": round(mine[n] / per_op_ms[n] / 1e6, 1),
                  "frac": round(mine[n] / per_op_ms[n] / 1e6 / peak, 3), "bytes": mine[n],
                  "share": round(per_op_ms[n] / step_sum, 3)} for n in names}
    traffic = TRAFFIC_PER_ROW["70b"].get(dom)
    line = {
        "metric": METRIC, "value": round(total_bytes / (ms / 1e3) / 1e9, 1), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded, reference config distributions)",
        "config": {"workload": WORKLOAD, "tokens": NT, "seq_len": SEQ_LEN_70B,
                   "rows_per_gpu": R, "logit_rows_per_gpu": LR, "hidden": c.hidden,
                   "heads": [c.n_q_heads, c.n_kv_heads, c.head_dim],
                   "intermediate": c.intermediate, "vocab": c.vocab,
                   "table_rows_per_gpu": vhi - vlo, "activations": "bf16 (f32 arithmetic)",
                   "logits": "f32", "bytes_per_step": total_bytes,
                   "l2": f"inputs larger than L2: {sum(mine.values()) / 1e9:.2f} GB of distinct "
                         "buffers per step per GPU",
                   "parallelism": f"rows and vocab sharded x{world}; the embedding gather "
                                  "reads peers' table parts through NCCL symmetric memory"},
        "rows_per_s": round(NT / (ms / 1e3), 1),
        "per_op": per_op,
        "largest_share": dom,
        "limiter": {
            "op": dom, "share_of_step": round(per_op_ms[dom] / step_sum, 3),
            "why": LIMITER_NOTE.get(dom, "HBM bandwidth"),
            "with_n": ("the per-GPU rows shrink as 1/N while the gather's share read over "
                       "NVLink grows as (N-1)/N" if world > 1 else
                       "one GPU: the gather reads local HBM only")},
        "gather": {"in_step": "one kernel over NCCL symmetric memory "
                              "(tb_b200_embedding_sharded_window)",
                   "window_ms": round(win_ms, 4), "nccl_sendrecv_ms": round(nccl_ms, 4),
                   "ipc_p2p_ms": round(p2p_ms, 4),
                   "rows_per_gpu": R, "row_bytes": c.hidden * 2,
                   "algorithmic_bytes_per_gpu": mine["embedding"],
                   "nvlink_read_bytes_per_gpu_max": int(nvlink_bytes),
                   "window_nvlink_GBps": (round(nvlink_bytes / win_ms / 1e6, 1)
                                          if world > 1 else None),
                   "nccl_sendrecv_nvlink_GBps": (round(nvlink_bytes / nccl_ms / 1e6, 1)
                                                 if world > 1 else None),
                   "ipc_p2p_nvlink_GBps": (round(nvlink_bytes / p2p_ms / 1e6, 1)
                                           if world > 1 else None),
                   "bit_exact": verified,
                   "check": "window, send/recv and IPC outputs equal; sampled rows equal the "
                            "table rows"},
        "roofline": {"bound": "hbm", "kernel": dom, "achieved": round(achieved, 1),
                     "peak": peak, "peak_source": peak_kind, "unit": "GB/s",
                     "frac": round(achieved / peak, 3),
                     "traffic": round(traffic * (LR if dom in ("softmax", "argmax") else R))
                     if traffic else None,
                     "algorithmic_bytes": mine[dom],
                     "traffic_source": TRAFFIC_SOURCE if traffic else
                     "no ncu capture of this kernel at this shape"},
        "e2e": {"value": round(total_bytes / (e2e_ms / 1e3) / 1e9, 2), "unit": "GB/s",
                "ms_per_step": round(e2e_ms, 3), "h2d_bytes_per_step": int(bi),
                "d2h_bytes_per_step": int(bo),
                "api": f"tb_b200_* C ABI: sharded gather from host ids, then {nb} row blocks "
                       f"on {len(streams)} streams with pinned host copies in and out"},
        "gpu_launches": int(launches),
        "clocks": clocks.summary(),
    }
    return line


# ------------------------------------------------------- bandwidth sweep
SWEEP_ROWS = [1 << k for k in range(10, 21)]
SWEEP_WIDTHS = [2048, 4096, 8192, 16384]
SWEEP_LOGIT_ROWS = [1, 16, 256, 4096]
SWEEP_VOCAB = 128256
SWEEP_REPS = 5  # timed launches per point (at least; --steps raises it, up to 20)


def run_sweep(args, rank, world, local):
    """Each point launched alone: residual+RMSNorm [rows, w] and SwiGLU over
    [rows, w] elements for the sweep's rows and widths, f32 and bf16, then
    softmax and argmax over [rows, 128256] f32 logits.  A point's rows are
    split over the ranks (tb_b200_partition); its time is the median over
    max(SWEEP_REPS, min(--steps, 20)) launches, after --warmup untimed ones,
    of the max over ranks.  L2 is flushed (a 512 MB
    write) before every timed launch whose buffers would fit in 4x L2.
    Points whose buffers exceed the memory budget are listed as skipped."""
    import torch
    import torch.distributed as dist
    import tb_b200 as T

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    L = T.lib()
    props = torch.cuda.get_device_properties(dev)
    budget = min(int(0.75 * props.total_memory), 136 * 10**9)
    l2 = getattr(props, "L2_cache_size", 126 * 2**20)
    flush = torch.empty(512 * 2**20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()
    sp = C.c_void_p(stream.cuda_stream)
    peak, peak_kind = peaks()
    g = torch.Generator(device=dev)
    g.manual_seed(777 + rank)

    def max_over_ranks(v):
        if world == 1:
            return v
        x = torch.tensor([float(v)], dtype=torch.float64, device=dev)
        dist.all_reduce(x, op=dist.ReduceOp.MAX)
        return float(x.item())

    reps = max(SWEEP_REPS, min(args.steps, 20))

    def time_point(launch, footprint):
        for _ in range(args.warmup):
            launch()
        times = []
        for _ in range(reps):
            if footprint < 4 * l2:
                flush.fill_(1)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            launch()
            b.record(stream)
            b.synchronize()
            times.append(max_over_ranks(a.elapsed_time(b)))
        return statistics.median(times)

    points, total_b, total_ms = [], 0, 0.0
    l0 = L.tb_b200_launch_count()
    uuid = getattr(props, "uuid", None)
    uuid = f"GPU-{uuid}" if uuid is not None else None
    with ClockSampler(local, uuid) as clocks:
        for dt, s_, tdt in ((T.F32, 4, torch.float32), (T.BF16, 2, torch.bfloat16)):
            for op in ("residual_rms_norm", "swiglu"):
                for w in SWEEP_WIDTHS:
                    for rows in SWEEP_ROWS:
                        lo, hi = T.partition(rows, world, rank)
                        big = -(-rows // world)  # the largest rank's rows
                        nt = 4 if op == "residual_rms_norm" else 3
                        pt = {"op": op, "dtype": "f32" if s_ == 4 else "bf16", "rows": rows,
                              "width": w}
                        if nt * big * w * s_ > budget:
                            pt["skipped"] = "buffers exceed the memory budget"
                            points.append(pt)
                            continue
                        r = hi - lo
                        buf = [torch.empty((r, w), dtype=tdt, device=dev).normal_(generator=g)
                               for _ in range(nt)]
                        if op == "residual_rms_norm":
                            gam = torch.empty((w,), dtype=tdt, device=dev).normal_(
                                1.0, 0.1, generator=g)
                            x, res, h, y = buf

                            def launch():
                                T.check(L.tb_b200_residual_rms_norm(
                                    dt, r, w, T.ptr(x), T.ptr(res), T.ptr(gam), T.ptr(h),
                                    T.ptr(y), C.c_float(1e-5), sp), "residual_rms_norm")
                            nbytes = W.bytes_res_rms(rows, w, s_)
                        else:
                            gate, up, out = buf

                            def launch():
                                T.check(L.tb_b200_swiglu(dt, r * w, T.ptr(gate), T.ptr(up),
                                                         T.ptr(out), sp), "swiglu")
                            nbytes = W.bytes_swiglu(rows, w, s_)
                        ms = time_point(launch, nt * r * w * s_)
                        del buf, launch
                        if op == "residual_rms_norm":
                            del x, res, h, y
                        else:
                            del gate, up, out
                        torch.cuda.empty_cache()
                        pt.update({"ms": round(ms, 5), "GB/s": round(nbytes / ms / 1e6, 1),
                                   "frac": round(nbytes / ms / 1e6 / peak, 3)})
                        points.append(pt)
                        total_b += nbytes
                        total_ms += ms
        for op in ("softmax", "argmax"):
            for rows in SWEEP_LOGIT_ROWS:
                lo, hi = T.partition(rows, world, rank)
                r = hi - lo
                x = torch.empty((r, SWEEP_VOCAB), device=dev).normal_(0.0, 3.0, generator=g)
                if op == "softmax":
                    y = torch.empty_like(x)

                    def launch():
                        T.check(L.tb_b200_softmax(T.F32, r, SWEEP_VOCAB, T.ptr(x), None,
                                                  T.ptr(y), sp), "softmax")
                    nbytes, fp = W.bytes_softmax(rows, SWEEP_VOCAB, 4), 2 * r * SWEEP_VOCAB * 4
                else:
                    y = torch.empty(max(r, 1), dtype=torch.int32, device=dev)

                    def launch():
                        T.check(L.tb_b200_argmax(T.F32, r, SWEEP_VOCAB, T.ptr(x), T.ptr(y), sp),
                                "argmax")
                    nbytes, fp = W.bytes_argmax(rows, SWEEP_VOCAB, 4), r * SWEEP_VOCAB * 4
                ms = time_point(launch, fp)
                del x, y, launch
                torch.cuda.empty_cache()
                points.append({"op": op, "dtype": "f32", "rows": rows, "width": SWEEP_VOCAB,
                               "ms": round(ms, 5), "GB/s": round(nbytes / ms / 1e6, 1),
                               "frac": round(nbytes / ms / 1e6 / peak, 3)})
                total_b += nbytes
                total_ms += ms
    launches = L.tb_b200_launch_count() - l0
    done = [p_ for p_ in points if "ms" in p_]
    biggest = max(done, key=lambda p_: p_["ms"])
    below = [f'{p_["op"]} {p_["dtype"]} {p_["rows"]}x{p_["width"]}: {p_["frac"]}'
             for p_ in done if p_["frac"] < 0.8]
    return {
        "metric": METRIC, "value": round(total_b / total_ms / 1e6, 1), "unit": "GB/s",
        "n_gpus": world, "steps": reps, "warmup": args.warmup,
        "ms_per_step": round(total_ms, 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32 and bf16 (f32 arithmetic)",
        "data": "synthetic (N(0,1) activations, N(0,3) logits)",
        "config": {"workload": WORKLOAD, "rows": SWEEP_ROWS, "widths": SWEEP_WIDTHS,
                   "logit_rows": SWEEP_LOGIT_ROWS, "vocab": SWEEP_VOCAB,
                   "memory_budget_bytes": budget,
                   "l2": "points smaller than 4x L2 flushed with a 512 MB write before each "
                         "timed launch; the rest exceed L2",
                   "parallelism": f"each point's rows split x{world}"},
        "points": points, "below_0.8": below,
        "roofline": {"bound": "hbm", "kernel": f'{biggest["op"]} {biggest["dtype"]} '
                                              f'{biggest["rows"]}x{biggest["width"]}',
                     "achieved": biggest["GB/s"], "peak": peak, "peak_source": peak_kind,
                     "unit": "GB/s", "frac": biggest["frac"], "traffic": None,
                     "traffic_source": "no ncu capture of the sweep"},
        "e2e": None,
        "gpu_launches": int(launches),
        "clocks": clocks.summary(),
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile-op", choices=["embedding", "layer_chain", "softmax", "argmax",
                                             "embedding_nccl", "embedding_ipc"],
                    help="only launch this op (warmup + steps times) on --rows rows: a small "
                         "case for ncu captures (70b: embedding is the symmetric-memory gather, "
                         "embedding_nccl the NCCL exchange, embedding_ipc the CUDA IPC kernel)")
    ap.add_argument("--config", choices=sorted(CONFIGS), default=DEFAULT_CONFIG,
                    help="70b (default): the Llama-70B prefill of 16384 tokens strong-scaled "
                         "over the ranks, with the vocab-sharded embedding gather and the "
                         "4096 x 128256 softmax/argmax; 7b: the Llama-7B prefill step on every "
                         "rank; decode: the 32-layer chain over a 256-sequence decode batch; "
                         "runner: single-sequence decode through the device TransformerRunner "
                         "(f32, 2:4); runner_int4: the same with INT4 projections; sweep: the "
                         "bandwidth sweep")
    ap.add_argument("--rows", type=int, default=None,
                    help="layer-op rows (70b: of the whole job; else per GPU; config's)")
    ap.add_argument("--logit-rows", type=int, default=None,
                    help="softmax/argmax rows (70b: of the whole job; 4096) -- for small ncu "
                         "captures")
    ap.add_argument("--runner-layers", type=int, default=RUNNER_LAYERS,
                    help="layers of the runner configs' model (32; fewer for small ncu captures)")
    args = ap.parse_args()
    global CFG, LOGIT_ROWS, WORKLOAD
    CFG, LOGIT_ROWS, WORKLOAD = CONFIGS[args.config]
    if args.logit_rows is not None:
        LOGIT_ROWS = args.logit_rows
    if args.rows is None:
        args.rows = CFG.rows
    args.warmup = max(args.warmup, 3)
    if args.profile_op in ("embedding_nccl", "embedding_ipc") and args.config != "70b":
        ap.error(f"--profile-op {args.profile_op} needs --config 70b")
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))

    if args.impl == "reference":
        if rank == 0:
            print(json.dumps(run_reference_runner(args, world)
                             if args.config in ("runner", "runner_int4")
                             else run_reference(args, world)))
        return

    import torch
    import torch.distributed as dist
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    try:
        decode = args.config == "decode"
        run = {"decode": run_decode, "runner": run_runner, "runner_int4": run_runner,
               "70b": run_sharded, "sweep": run_sweep}.get(args.config, run_gpu)
        line = run(args, rank, world, local)
        if line is None:
            return
        if rank == 0 and world == 1 and not args.no_cpu_baseline and args.config != "sweep":
            if args.config in ("runner", "runner_int4"):
                per_token, sample = cpu_sample_runner()
                line["cpu_baseline"] = {"value": round(1.0 / per_token, 4), "unit": "tokens/s",
                                        "cores": 1, "kind": "port", "sample": sample}
            else:
                line["cpu_baseline"] = cpu_baseline(
                    sample=cpu_sample_decode if decode else cpu_sample)
        if rank == 0:
            print(json.dumps(line))
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
