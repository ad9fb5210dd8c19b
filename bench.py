"""Benchmark of the quantized-matmul path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload prefill|square|decode]

Workloads (4-bit, group size 64, MLX affine layout, weights N(0, 0.02)
quantized with the min/max scheme, activations N(0, 1) in bf16, seeded):
  prefill  x [2048, 4096] . W[14336, 4096]^T   (the headline, TFLOP/s)
  square   x [2048, 4096] . W[4096, 4096]^T    (TFLOP/s)
  decode   x [1, 4096]    . W[4096, 4096]^T    (GB/s of algorithmic bytes)
  lmhead   x [1, 3072]    . W[128256, 3072]^T  (GB/s; a 4-bit tied LM head)
  sweep    14336x4096 and 4096x14336, bits 4/8, group 32/64/128, M 1..2048
           (one line of per-point times and roofline fractions)
A step is one quantized_matmul call through the C ABI.  Each rank runs its
own full step on its own GPU (token batches are independent: no collective on
the data path, weak scaling); the timed region is bracketed by a barrier and a
device synchronize, timed with CUDA events on the launching stream, and the
reported time is the max over ranks.  L2: every step reads a different one of
R input sets whose combined size is well above the 126 MB L2.

The line also carries: the decode (M=1) figure of the same run, the roofline
of the dominant kernel (CUDA-event duration per launch, algorithmic flops or
bytes, measured peaks), the CPU baseline (the oracle on the host cores, a
bounded sample of the same workload), the end-to-end figure through the
public API with host buffers (pinned host -> device copy of x, device -> host
copy of y inside the timed region), SM clocks sampled during the timed region,
and the number of this library's kernel launches in the timed region.

--impl reference runs the reference arm: the reference's CPU implementation of
this path is MLX, which cannot be built here, so the arm times the oracle's
restatement of it (oracle/nq_oracle.c) on all host threads; rank 0 only.
"""
import argparse
import json
import os
import statistics
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "4-bit g64 qmm: M=1 GB/s (% HBM peak), M=2048 TFLOP/s (% bf16 peak), 1–8 GPU"

WORKLOADS = {
    "prefill": dict(M=2048, N=14336, K=4096),
    "square": dict(M=2048, N=4096, K=4096),
    "decode": dict(M=1, N=4096, K=4096),
    "lmhead": dict(M=1, N=128256, K=3072),
}
BITS, GS = 4, 64
L2_BYTES = 126 * 1024 * 1024


def algo_bytes(M, N, K, bits=BITS, gs=GS):
    return N * K * bits // 8 + N * (K // gs) * 4 + M * K * 2 + M * N * 2


def algo_flops(M, N, K):
    return 2 * M * N * K


def peaks():
    p = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        d = json.load(open(path))
        p = {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
             "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
             "source": "measured"}
    return p


def ncu_traffic(workload):
    """DRAM bytes per launch of the dominant kernel from the committed ncu summary
    (profiles/traffic.txt: lines '<workload> <bytes per launch>'), or None."""
    path = os.path.join(ROOT, "profiles", "traffic.txt")
    if not os.path.exists(path):
        return None
    for line in open(path):
        parts = line.split()
        if len(parts) >= 2 and parts[0] == workload:
            return float(parts[1])
    return None


class ClockSampler:
    """SM clock and throttle reasons of one GPU, sampled every 5 ms by NVML from a
    background thread while the timed region runs."""

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.samples = []
        self.reasons = set()
        self.max_mhz = None
        self._stop = None
        self._thread = None

    def start(self):
        import threading
        try:
            import pynvml
            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.gpu)
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
        except Exception:
            return
        names = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
                 "sw_power_cap": 0x4}
        self._stop = threading.Event()

        def run():
            while not self._stop.is_set():
                try:
                    self.samples.append(float(pynvml.nvmlDeviceGetClockInfo(
                        h, pynvml.NVML_CLOCK_SM)))
                    r = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                    for n, bit in names.items():
                        if r & bit:
                            self.reasons.add(n)
                except Exception:
                    pass
                self._stop.wait(0.005)

        self._thread = threading.Thread(target=run, daemon=True)
        self._thread.start()

    def stop(self):
        if self._thread is None:
            return None
        self._stop.set()
        self._thread.join()
        if not self.samples:
            return None
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "samples": len(self.samples), "reasons": sorted(self.reasons),
                "source": "NVML, 5 ms period, during the timed region"}


def dist_setup(n_gpus):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(v, world):
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def make_inputs(M, N, K, sets, seed, bits=BITS, gs=GS):
    """R independent (x, W) sets quantized on the device (min/max scheme)."""
    import torch
    import neurons_b200 as nb
    g = torch.Generator(device="cuda").manual_seed(seed)
    out = []
    for _ in range(sets):
        w = torch.randn(N, K, device="cuda", generator=g) * 0.02
        wq, s, b = nb.quantize(w, gs, bits, nb.SCHEME_MINMAX)
        del w
        x = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
        y = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        out.append((x, wq, s, b, y))
    torch.cuda.synchronize()
    return out


def time_device(M, N, K, steps, warmup, world, seed, clocks=None, bits=BITS, gs=GS):
    """Device-resident inputs.  Returns (seconds for `steps` launches, max over
    ranks; mean seconds per launch on this rank; input sets used).

    Prefill-size steps are launched from the host one by one (the host runs far
    ahead of 0.1 ms kernels).  Decode-size steps (a few microseconds) are
    captured in one CUDA graph of `steps` launches and replayed, so that host
    submission is not part of what is timed -- the same way a decode loop
    replays a captured step."""
    import torch
    import neurons_b200 as nb
    per_set = algo_bytes(M, N, K, bits, gs) + M * N * 2
    sets = max(2, -(-3 * L2_BYTES // per_set))
    sets = min(sets, 64)
    data = make_inputs(M, N, K, sets, seed, bits, gs)
    stream = torch.cuda.current_stream()
    for i in range(warmup):
        x, wq, s, b, y = data[i % sets]
        nb.quantized_matmul(x, wq, s, b, True, gs, bits, out=y)
    torch.cuda.synchronize()
    graph = None
    if M <= 32:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for i in range(steps):
                x, wq, s, b, y = data[i % sets]
                nb.quantized_matmul(x, wq, s, b, True, gs, bits, out=y)
        for _ in range(max(1, warmup // steps + 1)):
            graph.replay()
        torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    if clocks is not None:
        clocks.start()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    if graph is not None:
        graph.replay()
    else:
        for i in range(steps):
            x, wq, s, b, y = data[i % sets]
            nb.quantized_matmul(x, wq, s, b, True, gs, bits, out=y)
    t1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop() if clocks is not None else None
    barrier(world)
    total = t0.elapsed_time(t1) / 1e3
    assert nb.take_device_error() == 0
    del graph
    return max_over_ranks(total, world), total / steps, sets, clk


def time_e2e(M, N, K, steps, warmup, world, seed):
    """Through the public API with host buffers: every step copies its own x from
    pinned host memory to the device, runs quantized_matmul and copies its own y
    back to pinned host memory.  The copies are pipelined the way a serving loop
    would run them: two device buffers for x and for y, the host->device copies
    on one copy stream and the device->host copies on another, so step i+1's
    input and step i-1's output cross PCIe while step i computes.  Every copy of
    every step is inside the timed region, which ends when the last step's y
    has reached host memory."""
    import torch
    import neurons_b200 as nb
    data = make_inputs(M, N, K, 1, seed + 1)
    _, wq, s, b, _ = data[0]
    gen = torch.Generator().manual_seed(seed)
    xh = [torch.randn(M, K, generator=gen).to(torch.bfloat16).pin_memory() for _ in range(2)]
    yh = [torch.empty(M, N, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    xd = [torch.empty(M, K, device="cuda", dtype=torch.bfloat16) for _ in range(2)]
    yd = [torch.empty(M, N, device="cuda", dtype=torch.bfloat16) for _ in range(2)]
    compute = torch.cuda.current_stream()
    h2d, d2h = torch.cuda.Stream(), torch.cuda.Stream()
    ev = lambda: torch.cuda.Event()
    x_ready = [ev(), ev()]     # x[j] on the device
    x_free = [ev(), ev()]      # the GEMM that read xd[j] finished
    y_ready = [ev(), ev()]     # the GEMM that wrote yd[j] finished
    y_free = [ev(), ev()]      # yd[j] copied out
    for j in range(2):
        x_free[j].record(compute)
        y_free[j].record(compute)

    def run(n):
        start = ev()
        start.record(compute)  # the copy streams start after the region's start event
        h2d.wait_event(start)
        d2h.wait_event(start)
        for i in range(n):
            j = i % 2
            h2d.wait_event(x_free[j])
            with torch.cuda.stream(h2d):
                xd[j].copy_(xh[j], non_blocking=True)
            x_ready[j].record(h2d)
            compute.wait_event(x_ready[j])
            compute.wait_event(y_free[j])
            nb.quantized_matmul(xd[j], wq, s, b, True, GS, BITS, out=yd[j])
            x_free[j].record(compute)
            y_ready[j].record(compute)
            d2h.wait_event(y_ready[j])
            with torch.cuda.stream(d2h):
                yh[j].copy_(yd[j], non_blocking=True)
            y_free[j].record(d2h)
        done = ev()
        done.record(d2h)
        compute.wait_event(done)

    run(warmup)
    torch.cuda.synchronize()
    barrier(world)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(compute)
    run(steps)
    t1.record(compute)
    torch.cuda.synchronize()
    barrier(world)
    total = max_over_ranks(t0.elapsed_time(t1) / 1e3, world)
    return total, M * K * 2, M * N * 2


LLAMA3B = dict(hidden=3072, n_heads=24, n_kv=8, head_dim=128, inter=8192, layers=28,
               vocab=128256)


def time_replay(tokens, warmup, world, seed, clocks=None):
    """Llama-3.2-3B decode replay (28 layers x 7 projections + the 4-bit LM head,
    M=1): one CUDA graph holds one token's 197 quantized_matmul launches and is
    replayed `tokens` times.  The 1.8 GB of weights dwarf the L2, so every token
    reads them from HBM.  Returns (seconds, max over ranks; replay object)."""
    import torch
    import neurons_b200 as nb
    from neurons_b200.replay import LlamaDecodeReplay
    rp = LlamaDecodeReplay(**LLAMA3B, bits=BITS, group_size=GS, seed=seed)
    g = torch.Generator(device="cuda").manual_seed(seed)
    rp.x.copy_(torch.randn(rp.x.shape, device="cuda", generator=g).to(torch.bfloat16))
    rp.step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        rp.step()
    for _ in range(warmup):
        graph.replay()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    barrier(world)
    torch.cuda.synchronize()
    if clocks is not None:
        clocks.start()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(tokens):
        graph.replay()
    t1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop() if clocks is not None else None
    barrier(world)
    assert nb.take_device_error() == 0
    total = t0.elapsed_time(t1) / 1e3
    del graph
    return max_over_ranks(total, world), rp, clk


def time_llama_step(prompt, tokens, world, seed, pk):
    """The Llama decode step (nq_llama_*) at the Llama-3.2-3B dims, random
    4-bit g64 weights, tied 4-bit LM head: a prompt of `prompt` tokens, then
    `tokens` greedy tokens generated back to back on the device (each step
    reads the previous argmax; no host round trip), timed with CUDA events.
    Per token: the weights once (the algorithmic bytes of the replay) plus the
    KV cache read by attention (positions so far x layers x 2 x n_kv x
    head_dim bf16)."""
    import torch
    import neurons_b200 as nb
    from neurons_b200.llama import LlamaDecoder
    c = LLAMA3B
    cfg = dict(n_layers=c["layers"], hidden=c["hidden"], n_heads=c["n_heads"],
               n_kv_heads=c["n_kv"], head_dim=c["head_dim"], intermediate=c["inter"],
               vocab=c["vocab"], bits=BITS, group_size=GS, max_context=prompt + tokens + 32,
               rms_eps=1e-5, rope_theta=500000.0)
    g = torch.Generator(device="cuda").manual_seed(6000 + seed)

    def qw(n, k, std=0.02):
        w = torch.randn(n, k, device="cuda", generator=g) * std
        q = nb.quantize(w, GS, BITS, nb.SCHEME_MINMAX)
        del w
        return q

    H, I, V = c["hidden"], c["inter"], c["vocab"]
    nq_, nkv = c["n_heads"] * c["head_dim"], c["n_kv"] * c["head_dim"]
    ones = lambda: (1 + 0.1 * torch.randn(H, device="cuda", generator=g)).to(torch.bfloat16)
    weights = {"embed": qw(V, H, 1.0), "final_norm": ones(), "layers": []}
    for _ in range(c["layers"]):
        weights["layers"].append({"q": qw(nq_, H), "k": qw(nkv, H), "v": qw(nkv, H),
                                  "o": qw(H, nq_), "gate": qw(I, H), "up": qw(I, H),
                                  "down": qw(H, I), "input_norm": ones(), "post_norm": ones()})
    dec = LlamaDecoder(cfg, weights)
    ptoks = torch.randint(0, V, (prompt,), device="cuda", generator=g, dtype=torch.int32)
    out = torch.empty(tokens, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream()

    def timed(fn):
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        fn()
        t1.record(stream)
        torch.cuda.synchronize()
        return t0.elapsed_time(t1) / 1e3

    # steps launched from the host one after another (warm-up pass first)
    dec.prefill(ptoks, logits=False)
    dec.generate(8, out=out[:8])
    dec.reset()
    dec.prefill(ptoks, logits=False)
    sec_stream = timed(lambda: dec.generate(tokens, out=out))
    # the same steps replayed from a CUDA graph of 16 steps
    per_graph = 16
    dec.reset()
    dec.prefill(ptoks, logits=False)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        dec.generate(per_graph, out=out[:per_graph])
    torch.cuda.synchronize()
    sec = timed(lambda: [graph.replay() for _ in range(tokens // per_graph)])
    tokens_g = tokens // per_graph * per_graph
    del graph
    assert nb.take_device_error() == 0
    dec.close()
    layer_w = (nq_ + 2 * nkv) * H + nq_ * H + 3 * I * H
    wbytes = c["layers"] * (layer_w * BITS // 8 + layer_w // GS * 4) + V * H * BITS // 8 + \
        V * (H // GS) * 4
    kv_avg = c["layers"] * 2 * nkv * 2 * (prompt + tokens / 2)
    byts = wbytes + kv_avg
    return {"workload": f"Llama-3.2-3B decode step (28 layers, RMSNorm, RoPE, GQA attention over "
                        f"the KV cache, SwiGLU, tied 4-bit LM head, argmax), prompt {prompt}, "
                        f"{tokens} tokens generated on the device",
            "tokens_per_s": tokens_g / sec, "us_per_token": sec / tokens_g * 1e6,
            "algorithmic_bytes_per_token": byts,
            "gbs": byts * tokens_g / sec / 1e9,
            "frac": byts * tokens_g / sec / 1e9 / pk["hbm_gbs"],
            "note": f"steps replayed from a CUDA graph of {per_graph} steps; launched from the "
                    f"host one by one: {sec_stream / tokens * 1e6:.0f} us/token",
            "launches_per_token": 5 * c["layers"] + 4}


def replay_summary(t, tokens, rp, world, pk):
    byts = rp.algorithmic_bytes()
    gbs = world * byts * tokens / t / 1e9
    return {"workload": "Llama-3.2-3B decode replay: 28 layers x (q,k,v,o,gate,up,down) + "
                        "4-bit LM head, M=1, one CUDA graph per token",
            "unit": "GB/s", "value": gbs, "tokens_per_s": world * tokens / t,
            "us_per_token": t / tokens * 1e6, "frac": gbs / world / pk["hbm_gbs"],
            "algorithmic_bytes_per_token": byts, "launches_per_token": rp.launches_per_token(),
            "tokens": tokens}


QWEN3_MOE = dict(E=128, top_k=8, H=2048, I=768)


def moe_weights(E, H, I, gen):
    import torch
    import neurons_b200 as nb
    out = []
    for n, k in ((I, H), (I, H), (H, I)):
        w = torch.randn(E, n, k, device="cuda", generator=gen) * 0.02
        out.append(nb.quantize(w, GS, BITS, nb.SCHEME_MINMAX))
        del w
    return out


def time_moe(T, steps, warmup, world, seed, clocks=None):
    """Qwen3-30B-A3B MoE switch step (router + gate/up/down gather_qmm + SwiGLU +
    weighted sum) for T tokens.  Three weight sets (1 GB) rotate so experts are
    read from HBM; T <= 64 steps are captured in one CUDA graph.
    Returns (seconds for `steps` steps, max over ranks; algorithmic bytes and
    flops per step, averaged over the steps)."""
    import torch
    import neurons_b200 as nb
    E, k, H, I = (QWEN3_MOE[x] for x in ("E", "top_k", "H", "I"))
    g = torch.Generator(device="cuda").manual_seed(seed)
    sets = []
    for _ in range(3):
        gate, up, down = moe_weights(E, H, I, g)
        x = torch.randn(T, H, device="cuda", generator=g).to(torch.bfloat16)
        logits = torch.randn(T, E, device="cuda", generator=g).to(torch.bfloat16)
        ws = torch.empty(max(nb.moe_workspace_size(T, E, k, H, I), 1), dtype=torch.uint8,
                         device="cuda")
        idx = torch.empty(T, k, dtype=torch.int32, device="cuda")
        sc = torch.empty(T, k, dtype=torch.float32, device="cuda")
        y = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
        sets.append((x, logits, gate, up, down, ws, idx, sc, y))
    lib = nb.lib()

    def step(i):
        x, logits, gate, up, down, ws, idx, sc, y = sets[i % 3]
        nb.ops.check(lib.nq_moe_route(nb.ops._ptr(logits), T, E, k, nb.ops._ptr(idx),
                                      nb.ops._ptr(sc), nb.ops._stream()))
        nb.moe_switch(x, idx, sc, gate, up, down, GS, BITS, workspace=ws, out=y)

    for i in range(warmup):
        step(i)
    torch.cuda.synchronize()
    graph = None
    if T <= 64:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for i in range(steps):
                step(i)
        graph.replay()
        torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    barrier(world)
    torch.cuda.synchronize()
    if clocks is not None:
        clocks.start()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    if graph is not None:
        graph.replay()
    else:
        for i in range(steps):
            step(i)
    t1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop() if clocks is not None else None
    barrier(world)
    assert nb.take_device_error() == 0
    per_expert = sum(t.numel() * t.element_size() for t in sets[0][2] + sets[0][3] + sets[0][4]) // E
    byts = 0
    for i in range(steps):
        x, logits, gate, up, down, ws, idx, sc, y = sets[i % 3]
        touched = int(torch.unique(idx).numel())
        byts += touched * per_expert + T * H * 2 * 2 + T * E * 2
    byts /= steps
    flops = 2 * T * k * 3 * I * H
    total = t0.elapsed_time(t1) / 1e3
    del graph
    return max_over_ranks(total, world), byts, flops, clk


def time_quant(steps, warmup, world, seed, pk):
    """quantize (fp32 W -> codes + bf16 scales/biases, the MLX edge-snapped
    scheme) and dequantize (codes + scales/biases -> bf16 W) of the prefill
    weight [14336, 4096] at 4-bit g64.  Two rotating weight sets; every call
    reads or writes more than L2.  Algorithmic bytes: what the call must read
    and write once."""
    import torch
    import neurons_b200 as nb
    rows, K = WORKLOADS["prefill"]["N"], WORKLOADS["prefill"]["K"]
    g = torch.Generator(device="cuda").manual_seed(5000 + seed)
    ws = [torch.randn(rows, K, device="cuda", generator=g) * 0.02 for _ in range(2)]
    qs = [nb.quantize(w, GS, BITS, nb.SCHEME_MLX_AFFINE) for w in ws]
    out_q = [tuple(torch.empty_like(t) for t in q) for q in qs]
    out_w = torch.empty(rows, K, dtype=torch.bfloat16, device="cuda")
    packed = rows * K * BITS // 8 + rows * (K // GS) * 4
    res = {"workload": f"W [{rows},{K}], {BITS}-bit g{GS}"}
    t = _events_time(lambda i: nb.dequantize(*qs[i % 2], GS, BITS, out=out_w), steps, warmup,
                     world)
    b = packed + rows * K * 2
    res["dequantize"] = {"us_per_call": t / steps * 1e6, "gbs": b * steps / t / 1e9,
                         "frac": b * steps / t / 1e9 / pk["hbm_gbs"],
                         "algorithmic_bytes_per_call": b}
    t = _events_time(lambda i: nb.quantize(ws[i % 2], GS, BITS, nb.SCHEME_MLX_AFFINE,
                                           out=out_q[i % 2]), steps, warmup, world)
    b = packed + rows * K * 4
    res["quantize"] = {"us_per_call": t / steps * 1e6, "gbs": b * steps / t / 1e9,
                       "frac": b * steps / t / 1e9 / pk["hbm_gbs"],
                       "algorithmic_bytes_per_call": b}
    assert nb.take_device_error() == 0
    return res


def moe_summary(T, t, steps, byts, flops, world, pk):
    sec = t / steps
    d = {"T": T, "us_per_step": sec * 1e6, "gbs": world * byts / sec / 1e9,
         "tflops": world * flops / sec / 1e12, "algorithmic_bytes_per_step": byts,
         "flops_per_step": flops}
    d["frac_hbm"] = byts / sec / 1e9 / pk["hbm_gbs"]
    d["frac_tensor"] = flops / sec / 1e12 / pk["bf16_tflops"]
    return d


def _events_time(step, steps, warmup, world, graph=False, clocks=None):
    """Device time of `steps` calls of step(i), bracketed by a barrier and a
    synchronize, CUDA events on the current stream, max over ranks.  With
    graph=True the steps are captured in one CUDA graph and replayed, as a
    decode loop does, so host submission is not timed.  The multi-rank steps
    use it too: their ranks wait for one another inside every step (flag
    barriers, collectives), so without a graph any rank's host jitter (a
    launch delayed by another thread of the process) stalls all of them."""
    import torch
    for i in range(warmup):
        step(i)
    torch.cuda.synchronize()
    g = None
    if graph:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for i in range(steps):
                step(i)
        g.replay()
        torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    if clocks is not None:
        clocks.start()
    stream = torch.cuda.current_stream()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    if g is not None:
        g.replay()
    else:
        for i in range(steps):
            step(i)
    t1.record(stream)
    torch.cuda.synchronize()
    if clocks is not None:
        clocks.last = clocks.stop()
    barrier(world)
    del g
    return max_over_ranks(t0.elapsed_time(t1) / 1e3, world)


def time_tp(comm, M, N, K, steps, warmup, world, rank):
    """Tensor-parallel quantized matmul: this rank's N/world weight rows, the
    output columns all-gathered so every rank holds y [M, N] (strong scaling:
    the total work is fixed as ranks are added).  Three rotating input sets."""
    import torch
    import neurons_b200 as nb
    from neurons_b200 import dist
    _, rows = dist.tp_shard(N, world, rank)
    g = torch.Generator(device="cuda").manual_seed(1000 + rank)
    sets = []
    for _ in range(3):
        w = torch.randn(rows, K, device="cuda", generator=g) * 0.02
        wq, s, b = nb.quantize(w, GS, BITS, nb.SCHEME_MINMAX)
        del w
        x = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
        y = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        ws = torch.empty(max(dist.tp_workspace_size(M, N, world), 1), dtype=torch.uint8,
                         device="cuda")
        sets.append((x, wq, s, b, y, ws))

    def step(i):
        x, wq, s, b, y, ws = sets[i % 3]
        dist.tp_quantized_matmul(comm, x, wq, s, b, N, GS, BITS, out=y, workspace=ws)

    t = _events_time(step, steps, warmup, world, graph=True)
    assert nb.take_device_error() == 0
    return t


def time_ep(comm, T, steps, warmup, world, rank):
    """Expert-parallel Qwen3-30B-A3B switch step for T tokens in total: this
    rank routes its T/world tokens, holds E/world experts; dispatch (all-gather
    of tokens and routing), the shard's switch step, combine (reduce-scatter
    of fp32 partials).  Strong scaling.  Two rotating weight sets."""
    import torch
    import neurons_b200 as nb
    from neurons_b200 import dist
    E, k, H, I = (QWEN3_MOE[v] for v in ("E", "top_k", "H", "I"))
    _, ne = dist.ep_shard(E, world, rank)
    _, nt = dist.ep_token_shard(T, world, rank)
    g = torch.Generator(device="cuda").manual_seed(2000 + rank)
    sets = []
    for _ in range(2):
        W = []
        for n, kk in ((I, H), (I, H), (H, I)):
            w = torch.randn(ne, n, kk, device="cuda", generator=g) * 0.02
            W.append(nb.quantize(w, GS, BITS, nb.SCHEME_MINMAX))
            del w
        x = torch.randn(nt, H, device="cuda", generator=g).to(torch.bfloat16)
        logits = torch.randn(nt, E, device="cuda", generator=g).to(torch.bfloat16)
        sets.append((x, logits, W))
    ws = torch.empty(dist.ep_workspace_size(T, E, k, H, I, world), dtype=torch.uint8,
                     device="cuda")
    y = torch.empty(nt, H, dtype=torch.bfloat16, device="cuda")

    def step(i):
        x, logits, W = sets[i % 2]
        idx, sc = nb.moe_route(logits, k)
        dist.ep_moe_switch(comm, x, T, idx, sc, W[0], W[1], W[2], E, GS, BITS, workspace=ws,
                           out=y)

    t = _events_time(step, steps, warmup, world, graph=True)
    assert nb.take_device_error() == 0
    return t


def time_ep_fused(comm, T, steps, warmup, world, rank, arena_offset):
    """time_ep with the dispatch and the combine as an all-to-all over NVLink
    (peer stores into the symmetric arena) instead of NCCL collectives."""
    import torch
    import neurons_b200 as nb
    from neurons_b200 import dist
    E, k, H, I = (QWEN3_MOE[v] for v in ("E", "top_k", "H", "I"))
    _, ne = dist.ep_shard(E, world, rank)
    _, nt = dist.ep_token_shard(T, world, rank)
    g = torch.Generator(device="cuda").manual_seed(2500 + rank)
    sets = []
    for _ in range(2):
        W = []
        for n, kk in ((I, H), (I, H), (H, I)):
            w = torch.randn(ne, n, kk, device="cuda", generator=g) * 0.02
            W.append(nb.quantize(w, GS, BITS, nb.SCHEME_MINMAX))
            del w
        x = torch.randn(nt, H, device="cuda", generator=g).to(torch.bfloat16)
        logits = torch.randn(nt, E, device="cuda", generator=g).to(torch.bfloat16)
        sets.append((x, logits, W))
    ws = torch.empty(dist.ep_fused_workspace_size(T, E, k, H, I, world), dtype=torch.uint8,
                     device="cuda")
    y = torch.empty(nt, H, dtype=torch.bfloat16, device="cuda")

    def step(i):
        x, logits, W = sets[i % 2]
        idx, sc = nb.moe_route(logits, k)
        dist.ep_moe_switch_fused(comm, x, T, idx, sc, W[0], W[1], W[2], E, arena_offset, GS, BITS,
                                 workspace=ws, out=y)

    t = _events_time(step, steps, warmup, world, graph=True)
    assert nb.take_device_error() == 0 and comm.take_error() == 0
    return t


def time_tp_fused(comm, M, N, K, steps, warmup, world, rank, clocks=None):
    """time_tp with the all-gather fused into the kernel's stores (peer
    writes into the symmetric arena over NVLink)."""
    import torch
    import neurons_b200 as nb
    from neurons_b200 import dist
    _, rows = dist.tp_shard(N, world, rank)
    g = torch.Generator(device="cuda").manual_seed(3000 + rank)
    sets = []
    ybytes = (M * N * 2 + 255) // 256 * 256
    for i in range(3):
        w = torch.randn(rows, K, device="cuda", generator=g) * 0.02
        wq, s, b = nb.quantize(w, GS, BITS, nb.SCHEME_MINMAX)
        del w
        x = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
        sets.append((x, wq, s, b, comm.symmetric_tensor(i * ybytes, (M, N))))

    def step(i):
        x, wq, s, b, y = sets[i % 3]
        dist.tp_quantized_matmul_fused(comm, x, wq, s, b, N, y, GS, BITS)

    t = _events_time(step, steps, warmup, world, graph=True, clocks=clocks)
    assert nb.take_device_error() == 0 and comm.take_error() == 0
    return t


def time_e2e_tp(comm, M, N, K, steps, warmup, world, rank):
    """The tensor-parallel call end to end: every rank copies the step's x from
    pinned host memory (each rank needs all of x), runs its shard with the
    output pushed to every rank, and rank 0 copies the whole y back to pinned
    host memory (every rank holds all of y; the host reads one copy).  Copies
    are inside the timed region, one stream, max over ranks."""
    import torch
    import neurons_b200 as nb
    from neurons_b200 import dist
    _, rows = dist.tp_shard(N, world, rank)
    g = torch.Generator(device="cuda").manual_seed(4000 + rank)
    w = torch.randn(rows, K, device="cuda", generator=g) * 0.02
    wq, s, b = nb.quantize(w, GS, BITS, nb.SCHEME_MINMAX)
    del w
    xh = torch.randn(M, K, generator=torch.Generator().manual_seed(rank)).to(
        torch.bfloat16).pin_memory()
    yh = torch.empty(M, N, dtype=torch.bfloat16).pin_memory()
    xd = torch.empty(M, K, device="cuda", dtype=torch.bfloat16)
    y = comm.symmetric_tensor(0, (M, N))

    def step(i):
        xd.copy_(xh, non_blocking=True)
        dist.tp_quantized_matmul_fused(comm, xd, wq, s, b, N, y, GS, BITS)
        if rank == 0:
            yh.copy_(y, non_blocking=True)

    t = _events_time(step, steps, warmup, world)
    assert nb.take_device_error() == 0 and comm.take_error() == 0
    return t, M * K * 2, (M * N * 2 if rank == 0 else 0)


def tp_headline(M, N, K, steps, warmup, world, rank, local):
    """N > 1 headline: the prefill problem split over the ranks by weight rows,
    each rank's output columns pushed into every rank's y by the GEMM epilogue
    (strong scaling: the total work is that of one single-GPU step)."""
    from neurons_b200 import dist
    comm = dist.Comm()
    comm.symmetric_alloc(3 * ((M * N * 2 + 255) // 256 * 256))
    clk = ClockSampler(local)
    # a fresh arena: its peer mappings' first touches (remote TLB fills over
    # NVLink) are warmed up before the timed steps
    t = time_tp_fused(comm, M, N, K, steps, max(warmup, 10), world, rank, clocks=clk)
    n_e = min(steps, 50)
    t_e, h2d, d2h = time_e2e_tp(comm, M, N, K, n_e, warmup, world, rank)
    comm.close()
    return t, getattr(clk, "last", None), (t_e, n_e, h2d, d2h)


def sharded_summary(world, rank, pk, single=None):
    """The tensor- and expert-parallel configurations at this N (strong
    scaling), for the JSON line."""
    from neurons_b200 import dist
    comm = dist.Comm()
    M0, N0 = WORKLOADS["prefill"]["M"], WORKLOADS["prefill"]["N"]
    ep_off = 3 * ((M0 * N0 * 2 + 255) // 256 * 256)
    comm.symmetric_alloc(ep_off + dist.ep_fused_arena_size(2048, QWEN3_MOE["top_k"],
                                                           QWEN3_MOE["H"], world))
    out = {"note": "strong scaling: total work fixed, split over the ranks; TP: NCCL all-gather "
                   "or the fused push (peer stores from the kernel), EP: NCCL all-gather + "
                   "reduce-scatter, or the all-to-all over peer memory; decode steps replayed "
                   "from a CUDA graph; time = max over ranks"}
    M, N, K = WORKLOADS["prefill"]["M"], WORKLOADS["prefill"]["N"], WORKLOADS["prefill"]["K"]
    n = 30
    t = time_tp(comm, M, N, K, n, 3, world, rank)
    out["tp_prefill"] = {"workload": "x[2048,4096] . W[14336,4096]^T, rows split over ranks",
                         "us_per_step": t / n * 1e6,
                         "tflops": algo_flops(M, N, K) * n / t / 1e12}
    t = time_tp_fused(comm, M, N, K, n, 3, world, rank)
    out["tp_prefill_fused"] = {"workload": "as tp_prefill, columns pushed to every rank by the "
                                           "GEMM's own stores over NVLink (no all-gather)",
                               "us_per_step": t / n * 1e6,
                               "tflops": algo_flops(M, N, K) * n / t / 1e12}
    d = WORKLOADS["decode"]
    n = 200
    t = time_tp(comm, d["M"], d["N"], d["K"], n, 5, world, rank)
    out["tp_decode"] = {"workload": "x[1,4096] . W[4096,4096]^T, rows split over ranks",
                        "us_per_step": t / n * 1e6,
                        "gbs": algo_bytes(d["M"], d["N"], d["K"]) * n / t / 1e9}
    t = time_tp_fused(comm, d["M"], d["N"], d["K"], n, 5, world, rank)
    out["tp_decode_fused"] = {"workload": "as tp_decode, columns pushed by the GEMV's stores",
                              "us_per_step": t / n * 1e6,
                              "gbs": algo_bytes(d["M"], d["N"], d["K"]) * n / t / 1e9}
    n = 10
    t = time_ep(comm, 2048, n, 3, world, rank)
    E, k, H, I = (QWEN3_MOE[v] for v in ("E", "top_k", "H", "I"))
    out["ep_moe_T2048"] = {"workload": "Qwen3-30B-A3B switch step, T=2048, experts and tokens "
                                       "split over ranks",
                           "us_per_step": t / n * 1e6,
                           "tflops": 2 * 2048 * k * 3 * I * H * n / t / 1e12}
    t = time_ep_fused(comm, 2048, n, 3, world, rank, ep_off)
    out["ep_moe_T2048_fused"] = {"workload": "as ep_moe_T2048, tokens dispatched to the ranks "
                                             "holding their experts and partial sums returned by "
                                             "peer stores over NVLink (all-to-all, no NCCL)",
                                 "us_per_step": t / n * 1e6,
                                 "tflops": 2 * 2048 * k * 3 * I * H * n / t / 1e12}
    comm.close()
    # strong-scaling efficiency against the single-GPU step timed in this run:
    # t(1 GPU) / (N * t(N GPUs))
    single = single or {}
    for key, ref in (("tp_prefill", "prefill_us"), ("tp_prefill_fused", "prefill_us"),
                     ("ep_moe_T2048", "moe_T2048_us"), ("ep_moe_T2048_fused", "moe_T2048_us")):
        if ref in single and key in out:
            out[key]["efficiency"] = single[ref] / (world * out[key]["us_per_step"])
            out[key]["single_gpu_us"] = single[ref]
    # this rank's kernels: per prefill step the shard's quantized matmul (1 or 2
    # kernels) plus the layout kernel (NCCL) or plus the ready and finish kernels
    # (fused); one GEMV per decode step (plus ready and finish when fused); nine
    # kernels per expert-parallel step.  NCCL's own kernels are not counted.
    import neurons_b200 as nb
    q = nb.quantized_matmul_launches(M, dist.tp_shard(N, world, rank)[1], K, GS, BITS)
    # the all-to-all step: router, ready, dispatch, exchange, the shard's switch
    # step (count, scan, fill, group_rows, gate/up, down, combine), combined, final
    launches = 30 * (q + 1) + 30 * (q + 2) + 200 + 200 * 3 + 10 * 9 + 10 * 13
    return out, launches


class CpuSample:
    """The oracle's qmm on every host thread over all M tokens and a slice of the
    weight rows.  `calibrate` grows the slice until one call takes about
    target_s seconds (never more than the N rows of the workload); `time` then
    re-times that same call."""

    def __init__(self, M, N, K):
        import numpy as np
        from oracle import oracle as O
        self.O, self.np = O, np
        self.M, self.N, self.K = M, N, K
        self.rng = np.random.default_rng(0)
        self.threads = O.max_threads()
        self.x = O.f32_to_bf16(self.rng.standard_normal((M, K)).astype(np.float32))
        self.rows = 0
        self.w = None

    def _prepare(self, rows):
        np, O = self.np, self.O
        self.w = O.quantize((self.rng.standard_normal((rows, self.K)) * 0.02).astype(np.float32),
                            BITS, GS, O.SCHEME_MINMAX)
        self.rows = rows

    def time(self):
        wq, s, b = self.w
        t = time.perf_counter()
        self.O.qmm(self.x, wq, s, b, BITS, GS, nthreads=self.threads)
        return time.perf_counter() - t

    def calibrate(self, target_s):
        rows = 8 if self.M > 1 else 512
        while True:
            self._prepare(rows)
            dt = self.time()
            if dt >= min(0.5, target_s / 4) or rows >= self.N:
                break
            rows = min(self.N, rows * 4)
        if dt < target_s and rows < self.N:
            self._prepare(int(min(self.N, rows * target_s / dt)))
        return self

    def result(self, dt):
        return {"rows": self.rows, "seconds": dt, "threads": self.threads,
                "tflops": algo_flops(self.M, self.rows, self.K) / dt / 1e12,
                "gbs": algo_bytes(self.M, self.rows, self.K) / dt / 1e9}


def cpu_baseline(M, N, K, target_s=12.0):
    """One bounded sample of the workload on the host cores, ~target_s seconds."""
    smp = CpuSample(M, N, K).calibrate(target_s)
    return smp.result(smp.time())


def torch_cpu_baseline(M, N, K, target_s=5.0):
    """A second CPU figure: the whole workload as a dense bf16 matmul in torch on
    every host thread, y = x . dequant(W)^T with the weights dequantized once
    beforehand (by the oracle, outside the timed calls) -- what a CPU user
    without a quantized kernel would run.  Repeated until ~target_s seconds."""
    import numpy as np
    import torch
    from oracle import oracle as O
    rng = np.random.default_rng(1)
    wq, sc, bi = O.quantize((rng.standard_normal((N, K)) * 0.02).astype(np.float32), BITS, GS,
                            O.SCHEME_MINMAX)
    wh = O.dequantize(wq, sc, bi, BITS, GS)
    del wq, sc, bi
    x = O.f32_to_bf16(rng.standard_normal((M, K)).astype(np.float32))
    xt = torch.from_numpy(x.view(np.int16)).view(torch.bfloat16)
    wt = torch.from_numpy(wh.view(np.int16)).view(torch.bfloat16)
    threads = os.cpu_count() or 1
    prev = torch.get_num_threads()
    torch.set_num_threads(threads)
    try:
        y = xt @ wt.T  # warm-up
        n, t = 0, time.perf_counter()
        while True:
            y = xt @ wt.T
            n += 1
            dt = time.perf_counter() - t
            if dt >= target_s or n >= 100:
                break
    finally:
        torch.set_num_threads(prev)
    del y
    sec = dt / n
    return {"seconds_per_call": sec, "threads": threads, "calls": n,
            "tflops": algo_flops(M, N, K) / sec / 1e12, "gbs": algo_bytes(M, N, K) / sec / 1e9}


SWEEP_SHAPES = ((14336, 4096), (4096, 14336))
SWEEP_M = (1, 8, 32, 128, 512, 2048)


def time_sweep(steps, warmup, world, seed, pk):
    """The quantized-matmul sweep: N x K in {14336 x 4096, 4096 x 14336}, bits
    {4, 8}, group size {32, 64, 128}, M {1, 8, 32, 128, 512, 2048}; per point
    the time per call (device-resident inputs, rotating sets larger than L2,
    the same timing as the headline) and the fraction of its roofline,
    max(bytes / HBM peak, flops / bf16 peak) / time."""
    pts = []
    for N, K in SWEEP_SHAPES:
        for bits in (4, 8):
            for gs in (32, 64, 128):
                for M in SWEEP_M:
                    n = steps if M <= 32 else max(10, steps // 10)
                    _, per, _, _ = time_device(M, N, K, n, warmup, world, seed, bits=bits, gs=gs)
                    byts, flops = algo_bytes(M, N, K, bits, gs), algo_flops(M, N, K)
                    roof = max(byts / (pk["hbm_gbs"] * 1e9), flops / (pk["bf16_tflops"] * 1e12))
                    pts.append({"N": N, "K": K, "bits": bits, "gs": gs, "M": M,
                                "us": per * 1e6, "gbs": byts / per / 1e9,
                                "tflops": flops / per / 1e12, "frac": roof / per,
                                "bound": "hbm" if byts / (pk["hbm_gbs"] * 1e9) >=
                                flops / (pk["bf16_tflops"] * 1e12) else "tensor"})
    return {"workload": "sweep", "points": pts, "peaks": {"hbm_gbs": pk["hbm_gbs"],
                                                          "bf16_tflops": pk["bf16_tflops"]}}


def ours(args):
    import torch
    world, rank, local = dist_setup(args.gpus)
    import neurons_b200 as nb
    nb.lib()
    pk = peaks()
    if args.workload == "llama3b-decode":
        return ours_replay(args, world, rank, local, pk)
    if args.workload == "quant":
        # quantize and dequantize of the prefill weight alone
        q = time_quant(args.steps, args.warmup, world, rank, pk)
        if rank == 0:
            print(json.dumps({"workload": "quant", **q}), flush=True)
        return
    if args.workload == "sweep":
        sw = time_sweep(args.steps, args.warmup, world, rank, pk)
        if rank == 0:
            print(json.dumps(sw), flush=True)
        return
    if args.workload == "llama3b-step":
        # the decode step alone (--steps tokens after a 128-token prompt)
        ls = time_llama_step(128, args.steps, world, rank, pk)
        if rank == 0:
            print(json.dumps({"workload": "llama3b-step", **ls}), flush=True)
        return
    if args.workload.startswith("moe-"):
        return ours_moe(args, world, rank, local, pk)
    wl = WORKLOADS[args.workload]
    M, N, K = wl["M"], wl["N"], wl["K"]
    t_dev, per_launch, sets, clk = time_device(M, N, K, args.steps, args.warmup, world,
                                               seed=rank, clocks=ClockSampler(local))
    flops, byts = algo_flops(M, N, K), algo_bytes(M, N, K)
    per_call = nb.quantized_matmul_launches(M, N, K, GS, BITS)  # 2: split wave tail
    launches = args.steps * per_call
    if M > 1:
        value = world * flops * args.steps / t_dev / 1e12
        unit = "TFLOP/s"
        achieved = flops / per_launch / 1e12
        roof = {"bound": "tensor", "achieved": achieved, "peak": pk["bf16_tflops"],
                "unit": "TFLOP/s", "frac": achieved / pk["bf16_tflops"],
                "peak_source": pk["source"] + " (burst bf16 GEMM)",
                "algorithmic_flops_per_launch": flops}
    else:
        value = world * byts * args.steps / t_dev / 1e9
        unit = "GB/s"
        achieved = byts / per_launch / 1e9
        roof = {"bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
                "frac": achieved / pk["hbm_gbs"], "peak_source": pk["source"],
                "algorithmic_bytes_per_launch": byts}
    roof["traffic"] = ncu_traffic(args.workload)
    # one call = the whole-tile grid, plus a clustered tail kernel when the last
    # wave is split; "achieved" is per call
    roof["kernels_per_call"] = per_call
    if args.kernel_only:
        if rank == 0:
            print(json.dumps({"workload": args.workload, "value": value, "unit": unit,
                              "roofline": roof, "clocks": clk}), flush=True)
        return
    line = {"metric": METRIC, "value": value, "unit": unit, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": t_dev / args.steps * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,0.02) weights quantized 4-bit g64, N(0,1) bf16 x)",
            "config": {"workload": args.workload, "M": M, "N": N, "K": K, "bits": BITS,
                       "group_size": GS, "parallelism": f"replicas x{world} (token batches)",
                       "l2": f"rotating {sets} input sets of "
                             f"{(algo_bytes(M, N, K) + M * N * 2) / 2**20:.0f} MiB (> L2)"},
            "roofline": roof, "gpu_launches": launches, "clocks": clk}
    tp_e2e = None
    if world > 1 and args.workload == "prefill":
        # strong scaling of the one problem; the replicas figure moves aside
        t_tp, clk_tp, tp_e2e = tp_headline(M, N, K, args.steps, args.warmup, world, rank, local)
        from neurons_b200 import dist
        q = nb.quantized_matmul_launches(M, dist.tp_shard(N, world, rank)[1], K, GS, BITS)
        line["replicas"] = {"value": value, "unit": unit, "scaling": "weak",
                            "ms_per_step": t_dev / args.steps * 1e3,
                            "parallelism": f"replicas x{world} (independent token batches)",
                            "roofline": roof}
        per_step = t_tp / args.steps
        line["value"] = flops / per_step / 1e12
        line["ms_per_step"] = per_step * 1e3
        line["scaling"] = "strong"
        line["config"]["parallelism"] = (
            f"tp{world}: weight rows split over the ranks, each rank's output columns "
            "pushed into every rank's y by its GEMM epilogue over NVLink (peer stores)")
        line["tp_efficiency"] = (t_dev / args.steps) / (world * per_step)
        share = flops / world / per_step / 1e12
        line["roofline"] = {"bound": "tensor", "achieved": share, "peak": pk["bf16_tflops"],
                            "unit": "TFLOP/s", "frac": share / pk["bf16_tflops"],
                            "peak_source": pk["source"] + " (burst bf16 GEMM)",
                            "algorithmic_flops_per_launch": flops // world,
                            "note": "this rank's share of the flops over the whole step (its "
                                    "GEMM, the ready/finish handshakes and the pushes)",
                            "traffic": None, "kernels_per_call": q + 2}
        line["clocks"] = clk_tp
        line["gpu_launches"] += args.steps * (q + 2)
    if args.workload != "decode" and not args.no_decode:
        d = WORKLOADS["decode"]
        dsteps = 2000
        t_d, pl_d, _, _ = time_device(d["M"], d["N"], d["K"], dsteps, max(args.warmup, 10), world,
                                      seed=rank + 100)
        db = algo_bytes(d["M"], d["N"], d["K"])
        line["decode"] = {"workload": "decode M=1 N=K=4096", "unit": "GB/s",
                          "value": world * db * dsteps / t_d / 1e9,
                          "kernel_gbs": db / pl_d / 1e9, "frac": db / pl_d / 1e9 / pk["hbm_gbs"],
                          "us_per_launch": pl_d * 1e6, "algorithmic_bytes_per_launch": db}
        line["gpu_launches"] += dsteps
    if args.workload == "prefill" and not args.no_moe:
        moe = {"workload": "Qwen3-30B-A3B MoE switch step (E=128, top-8, H=2048, I=768), "
                           "router + gate/up/down + SwiGLU + weighted sum"}
        for T, n in ((1, 500), (64, 200), (2048, 20)):
            t_m, b_m, f_m, _ = time_moe(T, n, 3, world, seed=rank + 300 + T)
            moe[f"T{T}"] = moe_summary(T, t_m, n, b_m, f_m, world, pk)
            # router + (a few tokens: up, down-with-combine | grouped: count,
            # scan, fill, [group_rows on the tensor-core path], up, down, combine)
            P = T * QWEN3_MOE["top_k"]
            line["gpu_launches"] += n * (3 if P <= QWEN3_MOE["E"] else
                                         (8 if P >= 8 * QWEN3_MOE["E"] else 7))
        line["moe"] = moe
    if args.workload == "prefill" and not args.no_quant:
        line["quant"] = time_quant(50, 3, world, rank, pk)
        line["gpu_launches"] += 2 * 50
    if args.workload == "prefill" and not args.no_sharded:
        single = {"prefill_us": t_dev / args.steps * 1e6}
        if "moe" in line:
            single["moe_T2048_us"] = line["moe"]["T2048"]["us_per_step"]
        line["sharded"], n_sh = sharded_summary(world, rank, pk, single)
        line["gpu_launches"] += n_sh
    if args.workload == "prefill" and not args.no_decode:
        t_r, rp, _ = time_replay(50, 3, world, seed=rank + 200)
        line["llama3b_decode"] = replay_summary(t_r, 50, rp, world, pk)
        line["gpu_launches"] += 50 * rp.launches_per_token()
        del rp
        ls = time_llama_step(128, 128, world, rank, pk)
        line["llama3b_decode_step"] = ls
        line["gpu_launches"] += (3 * 128 + 8 + 2 * 128) * ls["launches_per_token"]
    if tp_e2e is not None:
        t_e, n_e, h2d, d2h = tp_e2e
        line["e2e"] = {"value": flops * n_e / t_e / 1e12, "unit": unit, "h2d_bytes_per_step": h2d,
                       "d2h_bytes_per_step": d2h,
                       "note": "tensor parallel: x copied in on every rank, y copied out from "
                               "rank 0, one stream"}
        line["gpu_launches"] += n_e * line["roofline"]["kernels_per_call"]
    else:
        t_e, h2d, d2h = time_e2e(M, N, K, min(args.steps, 50), args.warmup, world, seed=rank)
        e2e_val = world * (flops if M > 1 else byts) * min(args.steps, 50) / t_e / (
            1e12 if M > 1 else 1e9)
        line["e2e"] = {"value": e2e_val, "unit": unit, "h2d_bytes_per_step": h2d,
                       "d2h_bytes_per_step": d2h}
        line["gpu_launches"] += min(args.steps, 50) * per_call
    if rank == 0 and world == 1 and not args.no_cpu:
        cb = cpu_baseline(M, N, K)
        line["cpu_baseline"] = {
            "value": cb["tflops"] if M > 1 else cb["gbs"], "unit": unit, "cores": cb["threads"],
            "kind": "port",
            "sample": f"oracle qmm (fp64 accumulation) over all {M} tokens x {cb['rows']} of "
                      f"{N} weight rows, K={K}, {cb['seconds']:.1f} s"}
        tc = torch_cpu_baseline(M, N, K)
        line["cpu_baseline"]["torch_cpu_bf16"] = {
            "value": tc["tflops"] if M > 1 else tc["gbs"], "unit": unit, "cores": tc["threads"],
            "sample": f"torch bf16 x[{M},{K}] . W_hat[{N},{K}]^T on the whole workload, weights "
                      f"dequantized beforehand, {tc['calls']} calls of "
                      f"{tc['seconds_per_call'] * 1e3:.1f} ms"}
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


def ours_replay(args, world, rank, local, pk):
    """--workload llama3b-decode: the replay alone, value in GB/s of algorithmic
    bytes (weights + activations) per token."""
    import torch
    t, rp, clk = time_replay(args.steps, args.warmup, world, seed=rank,
                             clocks=ClockSampler(local))
    s = replay_summary(t, args.steps, rp, world, pk)
    byts = rp.algorithmic_bytes()
    roof = {"bound": "hbm", "achieved": byts * args.steps / t / 1e9, "peak": pk["hbm_gbs"],
            "unit": "GB/s", "frac": s["frac"], "peak_source": pk["source"],
            "algorithmic_bytes_per_launch": byts / rp.launches_per_token(),
            "note": "whole-token average over the 197 launches of one graph",
            "traffic": ncu_traffic("llama3b-decode")}
    # End to end: the token's input row from pinned host memory, the logits back.
    xh = torch.randn(rp.x.shape).to(torch.bfloat16).pin_memory()
    lh = torch.empty(rp.logits.shape, dtype=torch.bfloat16).pin_memory()
    stream = torch.cuda.current_stream()
    n_e = min(args.steps, 50)
    for _ in range(args.warmup):
        rp.x.copy_(xh, non_blocking=True)
        rp.step()
        lh.copy_(rp.logits, non_blocking=True)
    torch.cuda.synchronize()
    barrier(world)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(n_e):
        rp.x.copy_(xh, non_blocking=True)
        rp.step()
        lh.copy_(rp.logits, non_blocking=True)
    t1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    t_e = max_over_ranks(t0.elapsed_time(t1) / 1e3, world)
    line = {"metric": METRIC, "value": s["value"], "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": t / args.steps * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,0.02) weights quantized 4-bit g64, N(0,1) bf16 x)",
            "config": {"workload": "llama3b-decode", **LLAMA3B, "bits": BITS, "group_size": GS,
                       "tokens_per_s": s["tokens_per_s"], "us_per_token": s["us_per_token"],
                       "parallelism": f"replicas x{world}",
                       "l2": "1.8 GB of weights per token (> L2)"},
            "roofline": roof, "gpu_launches": args.steps * rp.launches_per_token()
            + n_e * rp.launches_per_token(), "clocks": clk,
            "e2e": {"value": world * byts * n_e / t_e / 1e9, "unit": "GB/s",
                    "h2d_bytes_per_step": rp.x.numel() * 2,
                    "d2h_bytes_per_step": rp.logits.numel() * 2,
                    "note": "eager launches (no graph), host copies inside the timed region"}}
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


def ours_moe(args, world, rank, local, pk):
    """--workload moe-<T>: the Qwen3-30B-A3B switch step alone for T tokens."""
    T = int(args.workload.split("-")[1])
    t, byts, flops, clk = time_moe(T, args.steps, args.warmup, world, seed=rank,
                                   clocks=ClockSampler(local))
    s = moe_summary(T, t, args.steps, byts, flops, world, pk)
    tensor = T * QWEN3_MOE["top_k"] >= 8 * QWEN3_MOE["E"]
    line = {"metric": METRIC, "value": s["tflops"] if tensor else s["gbs"],
            "unit": "TFLOP/s" if tensor else "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": t / args.steps * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": args.workload, **QWEN3_MOE, "T": T, "bits": BITS,
                       "group_size": GS, "l2": "3 rotating weight sets of 340 MB (> L2)"},
            "moe": s, "clocks": clk}
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


def reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    # The replay's CPU sample is its largest projection shape (gate/up, 3072 -> 8192).
    wl = WORKLOADS.get(args.workload, dict(M=1, N=8192, K=3072))
    M, N, K = wl["M"], wl["N"], wl["K"]
    # Each step re-times one bounded sample; the sample is sized so that the
    # whole run (warm-up included) takes about two and a half minutes.
    per_step = min(4.0, max(0.1, 150.0 / (args.steps + args.warmup)))
    smp = CpuSample(M, N, K).calibrate(per_step)
    samples = []
    for i in range(args.warmup + args.steps):
        dt = smp.time()
        if i >= args.warmup:
            samples.append(smp.result(dt))
    cb = samples[-1]
    unit = "TFLOP/s" if M > 1 else "GB/s"
    v = statistics.mean(c["tflops"] if M > 1 else c["gbs"] for c in samples)
    sec = statistics.mean(c["seconds"] for c in samples)
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": unit, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic", "config": {"workload": args.workload, "M": M, "N": N, "K": K,
                                            "bits": BITS, "group_size": GS},
            "cpu_baseline": {"value": v, "unit": unit, "cores": cb["threads"], "kind": "port",
                             "sample": f"each step: oracle qmm over all {M} tokens x "
                                       f"{cb['rows']} of {N} weight rows, K={K} (the "
                                       "reference's MLX CPU path cannot be built here)"},
            "e2e": {"value": v, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="prefill", choices=sorted(WORKLOADS) + ["llama3b-decode", "llama3b-step",
                                                             "quant", "moe-1", "moe-64",
                                                             "moe-2048", "sweep"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-decode", action="store_true", help="skip the decode sub-lines")
    ap.add_argument("--no-moe", action="store_true", help="skip the MoE sub-line")
    ap.add_argument("--no-quant", action="store_true",
                    help="skip the quantize/dequantize sub-line")
    ap.add_argument("--no-sharded", action="store_true",
                    help="skip the tensor/expert-parallel sub-line")
    ap.add_argument("--kernel-only", action="store_true",
                    help="only the device-resident timed loop (a small target for ncu)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        reference(args)
    else:
        ours(args)


if __name__ == "__main__":
    main()
