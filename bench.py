"""MoE-layer tokens/s of the GGUF MoE block on B200 (benchmark config 4: a 48-layer stack of Qwen3-30B-A3B-shape
blocks, H=2048, E=128, top-8, F=768, Q4_0 weights, 16384 tokens), and the CPU reference arm.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python bench.py --decode            benchmark config 2 (decode batches 1 / 4 / 16 / 64, Q4_K), one line per batch
    python bench.py --config 3 | 5      benchmark config 3 (prefill, Q8_0, Zipf-skewed routing) or 5 (Qwen3-235B-A22B
                                        shape: H 4096, F 1536, Q4_0, 8192-token prefill and a 64-token decode batch)

One step = one forward of every layer of the stack over the step's token batch (the layers are independent blocks,
each with its own weights, all fed the same batch: the synthetic random weights would overflow bf16 through a chained
stack without the model's norms). value = tokens x layers / second over all ranks ("MoE-layer tokens/s").

Our arm: weights are generated on the GPU (seeded torch CUDA generator: fp16 d from |N(0, 0.02)|, nibbles uniform;
router fp32 N(0, 0.02); x bf16 N(0, 1)) and handed to the library as raw GGUF blocks; inputs resident in HBM before
the timed region; the weights stream from HBM each layer (340 MB a layer, far above the 126 MB L2, so no L2 flush is
needed). The timed region: W untimed steps, then K steps between CUDA events on the launching stream, a barrier and
a synchronize on both sides, the max over ranks. `e2e`: whole steps from pinned host memory to pinned host memory
(the step's tokens copied in, the layers through the C ABI, the last layer given the host output buffer: the library
copies the result back inside the call), inside the timed region. With N > 1 the block is expert-parallel:
rank r owns experts [r E / N, (r + 1) E / N) and T / N of the 16384 tokens; every layer exchanges token rows and
expert outputs over NCCL (artlite_b200/csrc/ep.cu): strong scaling (the total work is fixed).

`roofline`: the dominant kernel (the tcgen05 gate/up GEMM), its algorithmic FLOPs per launch (2 P H 2F, P = T K pairs)
over its average duration from CUDA events recorded between the forward's kernels on the forward's stream during the
timed steps, against the measured dense bf16 peak (MEASURED_PEAKS.json, sustained: a kernel inside a long step).
`cpu_baseline`: the reference's CPU path (its NumPy moe_ffn restated in oracle/moe_np.py, its compiled dequant_rows
and moe_route from oracle/_ref when they load here, else the C restatement) on a bounded token sample of one layer.

--impl reference: that CPU path alone, as the reference arm (rank 0; other ranks exit 0)."""

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

H, E, K, F = 2048, 128, 8, 768
LAYERS, TOKENS, QTYPE = 48, 16384, "Q4_0"
METRIC = "MoE-layer tokens/s, Qwen3-30B-A3B shape Q4_0, 1/2/4/8 B200; % of roofline"
UNIT = "tokens/s"
WORKLOAD = "qwen3-30b-a3b-moe-stack48-q4_0-t16384"


def measured_peaks() -> tuple[dict, str]:
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


# ---------------------------------------------------------------- clocks during the timed region

REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
           0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
           0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}


class Clocks:
    """nvidia-smi samples of the SM clock and throttle reasons every 50 ms, started before the warm-up (so that the
    sampler runs when the timed region starts); stop(t0, t1) keeps the samples taken within [t0, t1] (host time), or
    the one nearest to it when the region is shorter than the interval."""

    def __init__(self, gpu: int):
        self.gpu, self.proc, self.lines = gpu, None, []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), "--query-gpu=clocks.sm,clocks.max.sm,clocks_event_reasons.active",
                 "--format=csv,noheader,nounits", "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.time(), line.strip()))

    def stop(self, t0: float = 0.0, t1: float = float("inf")) -> dict:
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        rows = []
        for ts, ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 3:
                continue
            try:
                rows.append((ts, float(parts[0]), float(parts[1]), int(parts[2], 16)))
            except ValueError:
                continue
        inside = [r for r in rows if t0 <= r[0] <= t1]
        if not inside and rows:
            inside = [min(rows, key=lambda r: min(abs(r[0] - t0), abs(r[0] - t1)))]
        sm = [r[1] for r in inside]
        mx = max((r[2] for r in inside), default=0)
        reasons = set()
        for r in inside:
            for bit, name in REASONS.items():
                if r[3] & bit and name != "gpu_idle":
                    reasons.add(name)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx or None, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------- the CPU reference path

def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for ln in f:
                if ln.startswith("model name"):
                    return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


class CpuReference:
    """The reference's CPU path on one layer of the workload (T tokens): the router product, its routing (the
    reference's compiled moe_route from oracle/_ref when it loads here, else the C restatement), and ref.moe_ffn
    (restated in oracle/moe_np.py) with the compiled dequant_rows of the experts the tokens touch. The layer and the
    tokens are generated once; run() times one pass."""

    def __init__(self, T: int, seed: int = 0):
        from oracle import lib as olib
        from oracle import moe_np

        self.moe_np = moe_np
        ref = olib.reference()
        self.impl = ref if ref is not None else olib.oracle()
        self.kind = "reference" if ref is not None else "port"
        self.T = T
        self.layer, x, _ = moe_np.make_block(seed, T, qtype=QTYPE, H=H, E=E, F=F)
        self.xf = moe_np.bf16_to_f32(x)

    def run(self, blas_threads: int | None = None) -> float:
        from contextlib import nullcontext

        from threadpoolctl import threadpool_limits
        layer, impl = self.layer, self.impl

        def expert(e: int):
            return (impl.dequant_rows(QTYPE, layer.gate[e * F:(e + 1) * F], H),
                    impl.dequant_rows(QTYPE, layer.up[e * F:(e + 1) * F], H),
                    impl.dequant_rows(QTYPE, layer.down[e * H:(e + 1) * H], F))

        with threadpool_limits(blas_threads) if blas_threads else nullcontext():
            t0 = time.perf_counter()
            logits = self.xf @ layer.router.T
            ids, w = impl.route(logits, K)
            self.moe_np.moe_ffn(self.xf, ids, w, expert)
            return time.perf_counter() - t0


def blas_info() -> str:
    try:
        from threadpoolctl import threadpool_info
        return ", ".join(f"{i.get('internal_api')} {i.get('num_threads')} threads" for i in threadpool_info()) or "?"
    except ImportError:
        return "?"


def run_reference(args) -> None:
    """The reference arm: the reference's CPU path on the workload's own per-layer batch (T = --cpu-tokens, default
    the 16384 tokens of a layer of the stack), one layer per step, with all host cores; value = tokens x layers / s."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    ref = CpuReference(args.cpu_tokens, seed=1)
    for _ in range(args.warmup):
        ref.run()
    times = [ref.run() for _ in range(args.steps)]
    ms = 1000.0 * float(np.mean(times))
    value = ref.T / (ms / 1000.0)  # one layer per step
    sample = (f"{ref.T} tokens x 1 layer of the workload per step (router, routing, moe_ffn with the dequant of the "
              f"experts they touch); numpy BLAS ({blas_info()}) and the reference's dequant threads on all "
              f"{os.cpu_count()} host cores ({cpu_model()}); median step {1000.0 * float(np.median(times)):.1f} ms")
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded numpy: oracle.moe_np.make_block)",
            "config": {"workload": WORKLOAD, "tokens_per_step": ref.T, "layers_per_step": 1, "hidden": H,
                       "experts": E, "top_k": K, "expert_ffn": F, "qtype": QTYPE},
            "impl": "reference",
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": os.cpu_count(), "kind": ref.kind,
                             "sample": sample},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- our arm

def gen_layer(torch, g, dev):
    """One layer's raw Q4_0 tensors on the GPU: gate / up (E F rows of H), down (E H rows of F), router (E, H) fp32."""
    def q4_0(rows, cols):
        n = cols // 32
        raw = torch.empty((rows, n, 18), dtype=torch.uint8, device=dev)
        d = (torch.randn((rows, n), generator=g, device=dev) * 0.02).abs().half()
        raw[..., 0:2] = d.view(torch.uint8).view(rows, n, 2)
        raw[..., 2:] = torch.randint(0, 256, (rows, n, 16), dtype=torch.uint8, generator=g, device=dev)
        return raw.view(rows, n * 18)

    router = torch.randn((E, H), generator=g, device=dev) * 0.02
    return q4_0(E * F, H), q4_0(E * F, H), q4_0(E * H, F), router


def gen_layer_q4k(torch, g, dev):
    """One layer's raw Q4_K tensors on the GPU (144-byte super-blocks: d, dmin fp16 |N(0, 0.02)|, twelve bytes of
    uniform 6-bit scales / mins, 128 bytes of uniform nibbles) and the router (E, H) fp32."""
    def q4k(rows, cols):
        n = cols // 256
        raw = torch.randint(0, 256, (rows, n, 144), dtype=torch.uint8, generator=g, device=dev)
        for o in (0, 2):
            d = (torch.randn((rows, n), generator=g, device=dev) * 0.02).abs().half()
            raw[..., o:o + 2] = d.view(torch.uint8).view(rows, n, 2)
        return raw.view(rows, n * 144)

    router = torch.randn((E, H), generator=g, device=dev) * 0.02
    return q4k(E * F, H), q4k(E * F, H), q4k(E * H, F), router


def gen_q(torch, g, dev, qtype, rows, cols):
    """Raw GGUF rows of `qtype` on the GPU with the benchmark's distributions (fp16 scales |N(0, 0.02)|; Q4_0 nibbles
    uniform; Q8_0 int8 uniform -127..127)."""
    if qtype == "Q4_0":
        n = cols // 32
        raw = torch.empty((rows, n, 18), dtype=torch.uint8, device=dev)
        raw[..., 2:] = torch.randint(0, 256, (rows, n, 16), dtype=torch.uint8, generator=g, device=dev)
    elif qtype == "Q8_0":
        n = cols // 32
        raw = torch.empty((rows, n, 34), dtype=torch.uint8, device=dev)
        q = torch.randint(-127, 128, (rows, n, 32), dtype=torch.int16, generator=g, device=dev)
        raw[..., 2:] = q.to(torch.int8).view(torch.uint8)
    else:
        raise ValueError(qtype)
    d = (torch.randn((rows, n), generator=g, device=dev) * 0.02).abs().half()
    raw[..., 0:2] = d.view(torch.uint8).view(rows, n, 2)
    return raw.view(rows, -1)


def measure_config(config: int, layers: int, steps: int, warmup: int) -> list[dict]:
    """benchmark configs 3 and 5 on one GPU, `layers` layers of independent weights in turn (one dict per measured
    shape): tokens x layers / s, ms per layer, and the gate/up GEMM's share of the tensor roofline (tcgen05 path).
    The block's device status word is read after the timed steps (a bounded wait that ran out, or a bad expert id,
    raises)."""
    import torch
    from artlite_b200.moe.block import MoEBlock
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    if config == 3:
        h_, e_, k_, f_, qt, shapes = 2048, 128, 8, 768, "Q8_0", [("config3-prefill-q8_0-t4096-zipf1.1", 4096)]
    else:
        h_, e_, k_, f_, qt = 4096, 128, 8, 1536, "Q4_0"
        shapes = [("config5-prefill-q4_0-h4096-f1536-t8192", 8192), ("config5-decode-q4_0-h4096-f1536-b64", 64)]
    L = layers
    tmax = max(t for _, t in shapes)
    block = MoEBlock(hidden=h_, n_experts=e_, top_k=k_, expert_ffn=f_, max_tokens=tmax, n_layers=L, act_dtype="bf16",
                     device=0, path="auto")
    g = torch.Generator(device=dev)
    g.manual_seed(4000 + config)
    for layer in range(L):
        gate, up, down = gen_q(torch, g, dev, qt, e_ * f_, h_), gen_q(torch, g, dev, qt, e_ * f_, h_), \
            gen_q(torch, g, dev, qt, e_ * h_, f_)
        router = torch.randn((e_, h_), generator=g, device=dev) * 0.02
        block.set_weights(layer, gate=gate.data_ptr(), up=up.data_ptr(), down=down.data_ptr(),
                          router=router.data_ptr(), qtype=qt)
        if config == 3:  # the Zipf(1.1) expert skew: bias_e = -1.1 ln(rank_e), ranks a seeded permutation
            rank = torch.randperm(e_, generator=g, device=dev).float() + 1.0
            block.set_router_bias(layer, (-1.1 * torch.log(rank)).cpu().numpy().astype(np.float32))
        del gate, up, down, router
    torch.cuda.empty_cache()
    peaks, src = measured_peaks()
    stream = torch.cuda.Stream(device=dev)
    out = []
    for name, T in shapes:
        x = torch.randn((T, h_), generator=g, device=dev).to(torch.bfloat16)
        y = torch.empty((T, h_), dtype=torch.bfloat16, device=dev)

        def step():
            for layer in range(L):
                block.forward_ptr(x.data_ptr(), y.data_ptr(), T, layer=layer, stream=stream.cuda_stream)

        clocks = Clocks(0)
        clocks.start()
        with torch.cuda.stream(stream):
            for _ in range(warmup):
                step()
        torch.cuda.synchronize()
        t_host0 = time.time()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
        clk = clocks.stop(t_host0, time.time())
        block.sync()  # (the device status word: raises if a kernel reported an error)
        ms_layer = e0.elapsed_time(e1) / (steps * L)
        stages = np.array([block.stage_times(layer) for layer in range(L)])
        path = block.path(0)
        line = {"workload": name, "tokens": T, "hidden": h_, "experts": e_, "top_k": k_, "expert_ffn": f_, "qtype": qt,
                "ms_per_layer": ms_layer, "tokens_per_s": T / (ms_layer / 1000.0), "path": path, "layers": L,
                "steps": steps, "clocks": clk}
        if path == "tc" and stages.shape[1] >= 3:
            gu_ms = float(stages[:, 2].mean())
            flops = 2.0 * T * k_ * h_ * (2 * f_)
            peak = float(peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"]))
            line["roofline"] = {"kernel": "tc_expert_gemm gate/up (+ the gather)", "bound": "tensor",
                                "achieved": flops / (gu_ms / 1000.0) / 1e12, "peak": peak, "unit": "TFLOP/s",
                                "frac": flops / (gu_ms / 1000.0) / 1e12 / peak, "ms_per_launch": gu_ms,
                                "peak_source": f"{src} bf16_tflops_sustained"}
            down_ms = float(stages[:, 3].mean())
            layer_flops = flops * 1.5
            line["layer_roofline"] = {"bound": "tensor", "achieved": layer_flops / (ms_layer / 1000.0) / 1e12,
                                      "peak": peak, "unit": "TFLOP/s",
                                      "frac": layer_flops / (ms_layer / 1000.0) / 1e12 / peak,
                                      "down_frac": flops * 0.5 / (down_ms / 1000.0) / 1e12 / peak}
            line["stage_ms_mean"] = dict(zip(["router", "route+dispatch", "gather+gate_up", "down", "combine"],
                                             [float(v) for v in stages.mean(0)]))
        out.append(line)
    block.close()
    del block
    torch.cuda.empty_cache()
    return out


def run_config(args) -> None:
    for line in measure_config(args.config, args.layers, args.steps, args.warmup):
        print(json.dumps(line), flush=True)


# the reference's own MoE model's decode shape (Qwen3.6-35B-A3B, qwen35moe: 256 experts, top-8, FFN 512, a gated
# shared expert of FFN 512; tests/moe/ref.py:43-60)
QWEN35 = {"name": "qwen35moe", "H": 2048, "E": 256, "K": 8, "F": 512, "Fs": 512}
# the Q4_K_M layout of the reference's MoE files (Q4_K gate / up, Q6_K downs: tests/moe/test_prefill.py:1-5) at the
# benchmark's decode shape
Q4KM = {"name": "decode-q4_k_m", "H": 2048, "E": 128, "K": 8, "F": 768, "Fs": 0, "down": "Q6_K"}


def measure_decode(batches, layers: int, steps: int, warmup: int, path: str = "auto", shape: dict | None = None) -> list[dict]:
    """benchmark config 2 on one GPU: decode batches B = 1, 4, 16, 64 of the Q4_K block (bf16 x), each forward a CUDA
    graph, over `layers` layers in turn (their touched experts far exceed L2). One dict per B: tokens/s, and the
    HBM roofline of the bytes a forward must read (U touched experts x 2,654,208 B + the fp32 router 1,048,576 B).
    `shape` (H, E, K, F and a shared expert's Fs; "down": "Q6_K" for the Q4_K_M layout, Q4_K gate / up with Q6_K downs;
    "norm": each layer with its input norm and residual, artlite_moe_set_norm) measures another block shape the same
    way (the shared expert's rows and its gate vector are part of every forward's bytes). The block's device status
    word is read after the timed steps (raises on a kernel-reported error)."""
    import torch
    from artlite_b200.moe.block import MoEBlock
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    L = layers
    sh = shape or {"name": "decode-q4_k", "H": H, "E": E, "K": K, "F": F, "Fs": 0}
    h_, e_, k_, f_, fs = sh["H"], sh["E"], sh["K"], sh["F"], sh["Fs"]
    dq = sh.get("down", "Q4_K")
    block = MoEBlock(hidden=h_, n_experts=e_, top_k=k_, expert_ffn=f_, max_tokens=max(batches), n_layers=L,
                     act_dtype="bf16", device=0, path=path)
    g = torch.Generator(device=dev)
    g.manual_seed(3000)

    def q4k(rows, cols):
        n = cols // 256
        raw = torch.randint(0, 256, (rows, n, 144), dtype=torch.uint8, generator=g, device=dev)
        for o in (0, 2):
            d = (torch.randn((rows, n), generator=g, device=dev) * 0.02).abs().half()
            raw[..., o:o + 2] = d.view(torch.uint8).view(rows, n, 2)
        return raw.view(rows, n * 144)

    def q6k(rows, cols):  # (210-byte super-blocks: 192 bytes of uniform codes, int8 scales -32..31, d |N(0, 0.002)|)
        n = cols // 256
        raw = torch.randint(0, 256, (rows, n, 210), dtype=torch.uint8, generator=g, device=dev)
        sc = torch.randint(-32, 32, (rows, n, 16), dtype=torch.int16, generator=g, device=dev)
        raw[..., 192:208] = sc.to(torch.int8).view(torch.uint8)
        d = (torch.randn((rows, n), generator=g, device=dev) * 0.002).abs().half()
        raw[..., 208:210] = d.view(torch.uint8).view(rows, n, 2)
        return raw.view(rows, n * 210)

    for layer in range(L):
        gate, up = q4k(e_ * f_, h_), q4k(e_ * f_, h_)
        down = q6k(e_ * h_, f_) if dq == "Q6_K" else q4k(e_ * h_, f_)
        router = torch.randn((e_, h_), generator=g, device=dev) * 0.02
        block.set_weights(layer, gate=gate.data_ptr(), up=up.data_ptr(), down=down.data_ptr(),
                          router=router.data_ptr(), qtype="Q4_K", down_qtype=dq)
        if sh.get("norm"):  # (the layer's input norm and residual: y = x + moe(rms_norm(x, w)))
            wn = 1.0 + 0.1 * torch.randn((h_,), generator=g, device=dev)
            block.set_norm(layer, wn.data_ptr(), eps=1e-6, dtype="F32")
            del wn
        if fs:
            sg, su, sd = q4k(fs, h_), q4k(fs, h_), q4k(h_, fs)
            ginp = torch.randn((h_,), generator=g, device=dev) * 0.02
            block.set_shared(layer, gate=sg.data_ptr(), up=su.data_ptr(), down=sd.data_ptr(), ffn=fs, qtype="Q4_K",
                             gate_inp=ginp.data_ptr(), gate_dtype="F32")
            del sg, su, sd, ginp
        del gate, up, down, router
    torch.cuda.empty_cache()
    peaks, src = measured_peaks()
    stream = torch.cuda.Stream(device=dev)
    out = []
    for B in batches:
        x = torch.randn((B, h_), generator=g, device=dev).to(torch.bfloat16)
        y = torch.empty((B, h_), dtype=torch.bfloat16, device=dev)
        touched = []
        for layer in range(L):  # (the routing of each layer: its touched experts)
            block.forward_ptr(x.data_ptr(), y.data_ptr(), B, layer=layer, stream=stream.cuda_stream)
            block.sync()
            touched.append(len(np.unique(block.debug(B)["ids"])))
        clocks = Clocks(0)
        clocks.start()
        with torch.cuda.stream(stream):
            for _ in range(warmup):
                for layer in range(L):
                    block.forward_graph(x.data_ptr(), y.data_ptr(), B, layer=layer, stream=stream.cuda_stream)
        torch.cuda.synchronize()
        t_host0 = time.time()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            for layer in range(L):
                block.forward_graph(x.data_ptr(), y.data_ptr(), B, layer=layer, stream=stream.cuda_stream)
        e1.record(stream)
        torch.cuda.synchronize()
        clk = clocks.stop(t_host0, time.time())
        block.sync()  # (the device status word: raises if a kernel reported an error)
        ms_layer = e0.elapsed_time(e1) / (steps * L)
        U = float(np.mean(touched))
        per_expert = 2 * f_ * h_ * 144 // 256 + f_ * h_ * (210 if dq == "Q6_K" else 144) // 256  # (bytes per 256)
        nbytes = U * per_expert + e_ * h_ * 4 + (3 * fs * h_ * 144 // 256 + h_ * 4 if fs else 0) + \
            (h_ * 4 if sh.get("norm") else 0)
        gbs = nbytes / (ms_layer / 1000.0) / 1e9
        out.append({"workload": f"{sh['name']}-b{B}", "batch": B, "us_per_layer": ms_layer * 1000.0,
                    "tokens_per_s": B / (ms_layer / 1000.0), "experts_touched": U,
                    "roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                                 "frac": gbs / peaks["hbm_gbs"], "peak_source": f"{src} hbm_gbs",
                                 "bytes_per_layer": nbytes},
                    "path": block.path(0), "layers": L, "steps": steps, "clocks": clk})
    block.close()
    del block
    torch.cuda.empty_cache()
    return out


def run_decode(args) -> None:
    shape = QWEN35 if args.qwen35 else Q4KM if args.q4_k_m else None
    if args.norm:
        shape = dict(shape or {"name": "decode-q4_k", "H": H, "E": E, "K": K, "F": F, "Fs": 0}, norm=True)
        shape["name"] += "-norm"
    for line in measure_decode(args.batches, args.layers, args.steps, args.warmup, args.path, shape):
        print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--layers", type=int, default=LAYERS)
    ap.add_argument("--tokens", type=int, default=TOKENS)
    ap.add_argument("--cpu-tokens", type=int, default=TOKENS, help="tokens of a CPU reference pass (one layer)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="skip the decode sweep and config 3 of the default line")
    ap.add_argument("--decode", action="store_true", help="benchmark config 2 (decode batches, Q4_K) instead")
    ap.add_argument("--qwen35", action="store_true", help="with --decode: the qwen35moe shape (E 256, F 512, shared)")
    ap.add_argument("--q4-k-m", action="store_true", help="with --decode: Q4_K gate / up with Q6_K downs")
    ap.add_argument("--norm", action="store_true",
                    help="each layer with its input norm and residual (the default stack, or --decode)")
    ap.add_argument("--config", type=int, choices=[3, 5], help="benchmark config 3 or 5 (one GPU) instead")
    ap.add_argument("--path", default="auto", choices=["auto", "gemv", "tc"], help="expert path of --decode")
    ap.add_argument("--batches", type=int, nargs="+", default=[1, 4, 16, 64], help="decode batches of --decode")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
        return
    if args.decode:
        run_decode(args)
        return
    if args.config:
        if args.layers == LAYERS:
            args.layers = 4
        os.environ["ARTLITE_MOE_TIMING"] = "1"
        run_config(args)
        return

    os.environ["ARTLITE_MOE_TIMING"] = "1"  # per-stage CUDA events between the forward's kernels (no syncs)
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=300))

    from artlite_b200 import _lib
    from artlite_b200.moe.block import MoEBlock

    L = args.layers
    assert args.tokens % world == 0 and E % world == 0
    T = args.tokens // world  # this rank's tokens
    block = MoEBlock(hidden=H, n_experts=E, top_k=K, expert_ffn=F, max_tokens=T, n_layers=L, act_dtype="bf16",
                     device=local, path="auto", ep_rank=rank, ep_world=world)
    g = torch.Generator(device=dev)
    g.manual_seed(1000)  # the same weights on every rank (each keeps its own experts' rows)
    for layer in range(L):
        gate, up, down, router = gen_layer(torch, g, dev)
        block.set_weights(layer, gate=gate.data_ptr(), up=up.data_ptr(), down=down.data_ptr(),
                          router=router.data_ptr(), qtype=QTYPE)
        del gate, up, down, router
        if args.norm:  # (each layer with its input norm and residual: the reference's MoE layer in its decoder)
            wn = 1.0 + 0.1 * torch.randn((H,), generator=g, device=dev)
            block.set_norm(layer, wn.data_ptr(), eps=1e-6, dtype="F32")
            del wn
    torch.cuda.empty_cache()
    if world > 1:
        from artlite_b200.moe.block import ep_unique_id
        uid = [ep_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        block.ep_init(uid[0])
    g.manual_seed(2000 + rank)
    x = (torch.randn((T, H), generator=g, device=dev)).to(torch.bfloat16)
    ys = [torch.empty((T, H), dtype=torch.bfloat16, device=dev) for _ in range(2)]
    stream = torch.cuda.Stream(device=dev)

    def step():
        for layer in range(L):
            block.forward_ptr(x.data_ptr(), ys[layer & 1].data_ptr(), T, layer=layer, stream=stream.cuda_stream)

    def barrier():
        if world > 1:
            dist.barrier()

    clocks = Clocks(local)
    clocks.start()
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    t_host0 = time.time()
    launches0 = _lib.lib().artlite_moe_launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    t_host1 = time.time()
    launches = _lib.lib().artlite_moe_launch_count() - launches0
    block.sync()  # (the device status word of the timed steps: raises if a kernel reported an error)
    barrier()
    torch.cuda.synchronize()
    ms_total = e0.elapsed_time(e1)
    # per-stage times of every layer's forward in the last timed step (events on the forward's stream)
    stages = np.array([block.stage_times(layer) for layer in range(L)])
    path = block.path(0)
    clk = clocks.stop(t_host0, t_host1)
    t_max = torch.tensor([ms_total], device=dev)
    if world > 1:
        dist.all_reduce(t_max, op=dist.ReduceOp.MAX)
    ms_total = float(t_max.item())
    ms_step = ms_total / args.steps
    value = world * T * L / (ms_step / 1000.0)  # all ranks' tokens x layers per second

    # e2e: a step from pinned host memory to pinned host memory: the step's tokens copied to the device, the stack's
    # layers through the C ABI (the last one given the host y: the library copies the result back inside the call)
    e2e = None
    if not args.no_e2e:
        xh = torch.empty((T, H), dtype=torch.bfloat16, pin_memory=True)
        xh.copy_(x.cpu())
        yh = torch.empty((T, H), dtype=torch.bfloat16, pin_memory=True)
        xd = torch.empty_like(x)

        def step_host():
            with torch.cuda.stream(stream):
                xd.copy_(xh, non_blocking=True)
            for layer in range(L):
                y_ptr = yh.data_ptr() if layer == L - 1 else ys[layer & 1].data_ptr()
                block.forward_ptr(xd.data_ptr(), y_ptr, T, layer=layer, stream=stream.cuda_stream)

        step_host()
        torch.cuda.synchronize()
        barrier()
        t0 = time.perf_counter()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        n_e2e = max(1, min(args.steps, 3))
        for _ in range(n_e2e):
            step_host()
        ev1.record(stream)
        torch.cuda.synchronize()
        wall = (time.perf_counter() - t0) * 1000.0 / n_e2e
        dev_ms = ev0.elapsed_time(ev1) / n_e2e
        e_ms = torch.tensor([max(wall, dev_ms)], device=dev)
        if world > 1:
            dist.all_reduce(e_ms, op=dist.ReduceOp.MAX)
        e_ms = float(e_ms.item())
        e2e = {"value": world * T * L / (e_ms / 1000.0), "unit": UNIT, "h2d_bytes_per_step": T * H * 2,
               "d2h_bytes_per_step": T * H * 2, "ms_per_step": e_ms}

    # (every rank closes its block, then leaves the process group together)
    block.close()
    del block
    torch.cuda.empty_cache()
    barrier()
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return
    # the north star's other two targets, timed in the same run on one GPU: the decode batches (HBM roofline) and
    # the 4096-token Q8_0 prefill with Zipf-skewed routing (tensor roofline)
    extras = {}
    if world == 1 and not args.no_extras:
        extras["decode_sweep"] = {f"B{d['batch']}": {k: d[k] for k in ("us_per_layer", "tokens_per_s",
                                                                        "experts_touched", "roofline", "path",
                                                                        "layers", "steps", "clocks")}
                                  for d in measure_decode([1, 4, 16, 64], 8, 20, 3)}
        extras["qwen35moe_decode"] = {
            f"B{d['batch']}": {k: d[k] for k in ("us_per_layer", "tokens_per_s", "experts_touched", "roofline", "path",
                                                 "layers", "steps", "clocks")}
            for d in measure_decode([1, 16, 64], 8, 20, 3, shape=QWEN35)}
        extras["q4_k_m_decode"] = {
            f"B{d['batch']}": {k: d[k] for k in ("us_per_layer", "tokens_per_s", "experts_touched", "roofline", "path",
                                                 "layers", "steps", "clocks")}
            for d in measure_decode([1, 16, 64], 8, 20, 3, shape=Q4KM)}
        # the qwen35moe layer with its input norm and residual: the norm inside the first kernel that reads the rows,
        # and (ARTLITE_NORM_FUSE=0) the norm kernel first
        qn = dict(QWEN35, name="qwen35moe-norm", norm=True)
        extras["qwen35moe_decode_norm"] = {
            f"B{d['batch']}": {k: d[k] for k in ("us_per_layer", "tokens_per_s", "roofline", "path", "clocks")}
            for d in measure_decode([1, 16, 64], 8, 20, 3, shape=qn)}
        os.environ["ARTLITE_NORM_FUSE"] = "0"
        try:
            extras["qwen35moe_decode_norm_kernel"] = {f"B{d['batch']}": {"us_per_layer": d["us_per_layer"]}
                                                      for d in measure_decode([1, 16, 64], 8, 20, 3, shape=qn)}
        finally:
            del os.environ["ARTLITE_NORM_FUSE"]
        c3 = measure_config(3, 4, 10, 3)[0]
        extras["config3"] = {k: c3.get(k) for k in ("workload", "ms_per_layer", "tokens_per_s", "path", "roofline",
                                                    "layer_roofline", "stage_ms_mean", "layers", "steps", "clocks")}
    peaks, peak_src = measured_peaks()
    # stages (tc path): router, route+dispatch, gather + gate/up, down, combine
    roof = None
    if path == "tc" and stages.shape[1] >= 4 and world == 1:
        gu_ms = float(stages[:, 2].mean())
        P = T * K
        flops = 2.0 * P * H * (2 * F)
        achieved = flops / (gu_ms / 1000.0) / 1e12
        peak = float(peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"]))
        roof = {"kernel": "tc_expert_gemm<Q4_0, gate/up> (+ the dispatch gather, same stage)", "bound": "tensor",
                "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                "traffic": traffic_from_profiles(), "peak_source": f"{peak_src} bf16_tflops_sustained",
                "flops_per_launch": flops, "ms_per_launch": gu_ms}
    elif path == "tc" and stages.shape[1] >= 5:  # expert parallel: both expert GEMMs, the row exchange overlapped
        ex_ms = float((stages[:, 3] + stages[:, 4]).mean())
        P = T * K  # (a rank's experts process about as many rows as it dispatches)
        flops = 2.0 * P * H * (2 * F) + 2.0 * P * F * H
        achieved = flops / (ex_ms / 1000.0) / 1e12
        peak = float(peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"]))
        roof = {"kernel": "tc_expert_gemm<Q4_0> gate/up + down of a rank (its own rows, then the peers' in chunks, "
                          "the exchanges overlapped)", "bound": "tensor",
                "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                "traffic": None, "peak_source": f"{peak_src} bf16_tflops_sustained",
                "flops_per_launch": flops, "ms_per_launch": ex_ms}
    if world > 1:
        stage_names = ["router", "route+dispatch", "count exchange+gather", "own experts (rows in flight)",
                       "peer experts (chunks, exchanges overlapped)", "return exchange (rest)", "combine"]
    else:
        stage_names = ["router", "route+dispatch", "gather+gate_up", "down", "combine"] if path == "tc" else \
            ["router", "route+dispatch", "gate_up", "down", "combine"]
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(args.cpu_tokens)
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded torch CUDA generator: Q4_0 d=|N(0,0.02)| fp16, nibbles uniform; x bf16 N(0,1))",
            "config": {"workload": WORKLOAD + ("-norm" if args.norm else ""), "layers": L, "tokens": T * world,
                       "tokens_per_rank": T, "hidden": H,
                       "experts": E, "top_k": K, "expert_ffn": F, "qtype": QTYPE, "path": path,
                       "parallelism": f"ep{world}" if world > 1 else "single",
                       "l2": "inputs larger than L2 (340 MB of weights streamed per layer)"},
            "stage_ms_mean": dict(zip(stage_names, [float(v) for v in stages.mean(0)])),
            "roofline": roof, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": int(launches), "clocks": clk}
    line.update(extras)
    print(json.dumps(line), flush=True)


def traffic_from_profiles():
    """DRAM bytes per launch of the dominant kernel from the committed ncu summary, if there is one."""
    p = os.path.join(REPO, "profiles", "tc_expert_gemm_gu_q4_0.md")
    if not os.path.exists(p):
        return None
    for ln in open(p):
        if ln.startswith("traffic_bytes_per_launch:"):
            try:
                return float(ln.split(":", 1)[1].split()[0])
            except ValueError:
                return None
    return None


def cpu_baseline(T: int) -> dict:
    """The reference's CPU path on bounded samples (about 20-40 s of CPU work): the value is the median of three
    passes over one layer of the workload's own batch (T tokens) with all host cores; beside it, a 1024-token layer
    with all cores and with one BLAS thread (median of five each), where the dequant of the touched experts weighs
    more."""
    big = CpuReference(T, seed=50)
    big.run()  # (warm)
    t_big = [big.run() for _ in range(3)]
    small = CpuReference(1024, seed=51)
    small.run()
    t_all = [small.run() for _ in range(5)]
    t_one = [small.run(blas_threads=1) for _ in range(5)]
    value = T / float(np.median(t_big))
    return {"value": value, "unit": UNIT, "cores": os.cpu_count(), "kind": big.kind,
            "sample": f"median of 3 passes of {T} tokens x 1 layer (router, routing, moe_ffn with the dequant of the "
                      f"experts they touch), numpy BLAS on all cores ({blas_info()}), the reference's dequant "
                      f"threads; host {cpu_model()}",
            "cpu_model": cpu_model(),
            "t1024_all_cores_tokens_per_s": 1024 / float(np.median(t_all)),
            "t1024_one_blas_thread_tokens_per_s": 1024 / float(np.median(t_one))}


if __name__ == "__main__":
    main()
