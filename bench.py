#!/usr/bin/env python
"""Benchmark of the B200 row-op hot path (libtb_b200.so), one JSON line.

Workload: one pass of the per-token row ops of a Llama-7B-shape prefill of
4096 tokens -- the reference engine's layer ops batched over rows:
  embedding gather          ids [4096] -> rows of a [32000, 4096] table
  residual + RMSNorm        [4096, 4096]                    } one fused
  RoPE on Q and K           [4096, 32, 128] x 2, pos 0..4095 } layer-chain
  SwiGLU silu(gate)*up      [4096, 11008]                    } launch
  row softmax               logits [4096, 32000] f32
  greedy argmax             logits [4096, 32000] f32 (own buffer)
Activations bf16 (f32 arithmetic), logits f32; synthetic seeded inputs with
the reference config's distributions.  Every op reads distinct buffers and a
step moves ~2.2 GB, far more than the 126 MB L2, so nothing is served from
L2 across steps.

metric: algorithmic HBM bytes of the step (each input read once, each
output written once) / device time, in GB/s, over all ranks; rows/s beside
it.  --gpus N (torchrun) runs the same per-GPU workload on every rank (weak
scaling, no collective in the data path) and takes the max time over ranks.

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

# --config: the default is the Llama-7B prefill (the headline); 70b runs
# the Llama-70B prefill's layer ops on 16384 tokens and the bandwidth
# sweep's widest softmax/argmax point (4096 rows of 128256 logits).
CONFIGS = {
    "7b": (W.CONFIGS["7b"], None, "llama7b-prefill-4096 row ops (embedding, residual+RMSNorm, "
                                  "RoPE, SwiGLU, softmax, argmax)"),
    "70b": (W.CONFIGS["70b"], 4096, "llama70b-prefill-16384 layer ops (embedding, residual+RMSNorm, "
                                    "RoPE, SwiGLU) + softmax/argmax over 4096 x 128256 logits"),
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
CFG, LOGIT_ROWS, WORKLOAD = CONFIGS["7b"]
E2E_BLOCKS = 8    # row blocks of the end-to-end step
E2E_STREAMS = 3   # streams they are spread over
METRIC = "fused layer-op HBM GB/s"


def logit_rows(rows):
    """Rows of the softmax/argmax logits for `rows` layer-op rows."""
    return rows if LOGIT_ROWS is None else min(rows, LOGIT_ROWS)


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per row of each
# kernel, from one ncu capture each (profiles/*.md), for roofline.traffic.
# Writes still dirty in L2 when a kernel ends are not in the write count.
TRAFFIC_PER_ROW = {
    "embedding": (32137856 / 4096, "profiles/k_embed_llama7b-prefill-4096.md"),
    "layer_chain": (485573888 / 4096, "profiles/k_chain_llama7b-prefill-4096.md"),
    "softmax": ((192851456 + 74482944) / 1024, "profiles/k_softmax_staged_logits-1024x32000.md"),
    "argmax": (530358016 / 4096, "profiles/k_argmax_llama7b-prefill-4096.md"),
}


def step_bytes(rows, act_s):
    c = CFG
    lr = logit_rows(rows)
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
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
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
                     "traffic": round(TRAFFIC_PER_ROW["layer_chain"][0] * R),
                     "algorithmic_bytes": lb,
                     "traffic_source": TRAFFIC_PER_ROW["layer_chain"][1]
                                       + " (ncu, same row shape, scaled to the launch's rows)",
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
                     "traffic": (round(TRAFFIC_PER_ROW[dom][0] * (LR if dom in ("softmax", "argmax") else R))
                                 if CFG is CONFIGS["7b"][0] else None),
                     "algorithmic_bytes": parts[dom],
                     "traffic_source": (TRAFFIC_PER_ROW[dom][1] + " (ncu, scaled to the launch's rows)"
                                        if CFG is CONFIGS["7b"][0] else
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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile-op", choices=["embedding", "layer_chain", "softmax", "argmax"],
                    help="only launch this op (warmup + steps times) on --rows rows: a small "
                         "case for ncu captures")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="7b",
                    help="7b (default): the Llama-7B prefill step; 70b: the Llama-70B prefill's "
                         "layer ops and the sweep's 4096 x 128256 softmax/argmax; decode: the "
                         "32-layer chain over a 256-sequence decode batch; runner: single-"
                         "sequence decode through the device TransformerRunner (f32, 2:4); "
                         "runner_int4: the same with INT4 projections")
    ap.add_argument("--rows", type=int, default=None, help="layer-op rows per GPU (config's)")
    ap.add_argument("--runner-layers", type=int, default=RUNNER_LAYERS,
                    help="layers of the runner configs' model (32; fewer for small ncu captures)")
    args = ap.parse_args()
    global CFG, LOGIT_ROWS, WORKLOAD
    CFG, LOGIT_ROWS, WORKLOAD = CONFIGS[args.config]
    if args.rows is None:
        args.rows = CFG.rows
    args.warmup = max(args.warmup, 3)
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
        run = {"decode": run_decode, "runner": run_runner,
               "runner_int4": run_runner}.get(args.config, run_gpu)
        line = run(args, rank, world, local)
        if line is None:
            return
        if rank == 0 and world == 1 and not args.no_cpu_baseline:
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
