"""Benchmark of the GDN op on B200: BASELINE.json's metric on its config 1 (and config 3 as a side line).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one forward + backward of the gated delta rule at config 1 (B=8, T=4096, H=16, dk=dv=128,
bf16 activations, fp32 g and state, chunk 64) on synthetic seeded inputs with config 0's value
distributions. Under torchrun every rank runs its own B=8 shard (batch x head sharding, no collective:
weak scaling); the timed region is bracketed by barrier + synchronize on every rank and the time is the
max over ranks. Prints one JSON line on rank 0.

``value``: device-timed tokens/s with inputs resident in HBM (inputs total ~0.8 GB per rank, larger than
the 126 MB L2, so no flush is needed between steps). ``e2e``: the same step through the public API from
pinned host buffers (inputs copied in, outputs o/dq/dk/dv/dg/dbeta copied out, inside the timed region).
``--impl reference``: the reference algorithm on the host cores (the C restatement of
sore/model/gdn_ref.py in ``oracle/``; the Python reference itself is not present on the GPU box), rank 0.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

CFG1 = dict(B=8, T=4096, H=16, D=128)
CFG3 = dict(N=256, H=16, D=128)
METRIC = "GDN fwd+bwd tokens/s (B8 T4096 H16 d128 bf16); decode-step HBM GB/s"
C = 64
FWD_FLOP_PER_TOKEN_HEAD = 10 * C * 128 + 6 * 128 * 128 + C * C / 3  # chunked fwd count, 181,589
# What bounds the strong-scaling side line (the serial part of the step at few units per GPU).
STRONG_LIMITER = ("each (sequence, head) unit walks its 64 chunks serially in one CTA: with {units} units per "
                  "rank, {units} SMs work and the step time stays the per-unit chain time")
STRONG_LIMITER_PIECES = ("{units} units per rank, each cut into {P} pieces of {chunks} chunks: three state passes, "
                         "a dS-only sweep and a full sweep of {chunks} chunks per step (the pieces' maps and "
                         "end-state gradients), each still one CTA per piece walking its chunks serially")
PEAKS_FALLBACK = dict(hbm_gbs=6650.0, bf16_tflops=1590.0, bf16_tflops_sustained=1400.0)
# DRAM bytes (read + write) per launch from ncu captures of this build: the backward pass (the reverse-sweep
# launch over the records the forward saved) captured at batch 2 and scaled by 4 to batch 8; the decode step
# at full config-3 size.
BWD_PASS_TRAFFIC_BYTES = (319.8e6 + 83.8e6) * 4
DECODE_TRAFFIC_BYTES = 271.6e6 + 210.9e6


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return PEAKS_FALLBACK, "fallback"


def make_inputs(B, T, H, D, device, seed):
    import torch

    gen = torch.Generator(device=device).manual_seed(seed)
    q = torch.randn(B, T, H, D, device=device, generator=gen).bfloat16()
    k = torch.randn(B, T, H, D, device=device, generator=gen).bfloat16()
    v = torch.randn(B, T, H, D, device=device, generator=gen).bfloat16()
    g = torch.nn.functional.logsigmoid(torch.randn(B, T, H, device=device, generator=gen)) / 16
    beta = torch.sigmoid(torch.randn(B, T, H, device=device, generator=gen)).bfloat16()
    do = torch.randn(B, T, H, D, device=device, generator=gen).bfloat16()
    return dict(q=q, k=k, v=v, g=g, beta=beta, do=do)


class ClockSampler:
    """SM clock and throttle-reason sampling DURING the timed region, by polling NVML from a thread every
    ``period_s`` (a timed region of a few steps lasts tens of milliseconds, shorter than nvidia-smi's
    sampling interval). The GPU is found by the UUID torch reports for the CUDA device, so the index
    mapping under CUDA_VISIBLE_DEVICES does not matter."""

    REASONS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40), ("sw_thermal_slowdown", 0x20),
               ("sw_power_cap", 0x4), ("hw_power_brake_slowdown", 0x80))

    def __init__(self, device_index, period_s=0.002):
        self.device_index = device_index
        self.period_s = period_s
        self.samples = []  # (sm_mhz, reasons bitmask, power mW)
        self.max_mhz = None
        self.error = None
        self._stop = threading.Event()
        self._thread = None

    def __enter__(self):
        try:
            import pynvml
            import torch

            pynvml.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(self.device_index).uuid)
            self._nvml = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self._thread = threading.Thread(target=self._poll, daemon=True)
            self._thread.start()
        except Exception as e:  # no NVML: the line reports zero samples and the reason
            self.error = f"{type(e).__name__}: {e}"
        return self

    def _poll(self):
        nv, h = self._nvml, self._h
        while not self._stop.is_set():
            try:
                self.samples.append((nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM),
                                     nv.nvmlDeviceGetCurrentClocksEventReasons(h), nv.nvmlDeviceGetPowerUsage(h)))
            except Exception as e:
                self.error = f"{type(e).__name__}: {e}"
                return
            self._stop.wait(self.period_s)

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=5)

    def summary(self):
        if not self.samples:
            out = {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
            if self.error:
                out["error"] = self.error
            return out
        mask = 0
        for _, m, _ in self.samples:
            mask |= m
        return {"sm_mhz": statistics.median(s[0] for s in self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": [n for n, bit in self.REASONS if mask & bit], "samples": len(self.samples),
                "power_w": round(statistics.median(s[2] for s in self.samples) / 1e3, 1), "source": "nvml"}


def dist_setup(n_gpus):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return rank, world, local


def barrier(world):
    import torch
    import torch.distributed as dist

    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()


def max_over_ranks(x, world):
    import torch
    import torch.distributed as dist

    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def decode_bench(dev, rank, world, n_dec=1024, timed=True):
    """Decode (config 3): 256 sequences x 16 heads, fp32 state in HBM, bf16 token inputs; one step
    updates every state in place; 1,024 consecutive steps are timed, as config 3 specifies. Returns
    (ms per step, HBM bytes per step)."""
    import torch

    from sorernn_b200 import fused_recurrent_gated_delta_rule_step

    N, Hd, Dd = CFG3["N"], CFG3["H"], CFG3["D"]
    gen = torch.Generator(device=dev).manual_seed(99 + rank)
    state = torch.randn(N, Hd, Dd, Dd, device=dev, generator=gen) * 0.02
    dq = torch.nn.functional.normalize(torch.randn(N, Hd, Dd, device=dev, generator=gen), dim=-1).bfloat16()
    dk = torch.nn.functional.normalize(torch.randn(N, Hd, Dd, device=dev, generator=gen), dim=-1).bfloat16()
    dv = torch.randn(N, Hd, Dd, device=dev, generator=gen).bfloat16()
    dg = (torch.nn.functional.logsigmoid(torch.randn(N, Hd, device=dev, generator=gen)) / 16).bfloat16()
    db = torch.sigmoid(torch.randn(N, Hd, device=dev, generator=gen)).bfloat16()
    do_buf = torch.empty_like(dv)
    for _ in range(5):
        fused_recurrent_gated_delta_rule_step(dq, dk, dv, dg, db, state, out=do_buf)
    dec_bytes = 2 * state.numel() * 4 + 3 * dv.numel() * 2 + do_buf.numel() * 2 + 2 * dg.numel() * 2
    if not timed:
        for _ in range(n_dec):
            fused_recurrent_gated_delta_rule_step(dq, dk, dv, dg, db, state, out=do_buf)
        torch.cuda.synchronize(dev)
        return None, dec_bytes
    barrier(world)
    s3, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s3.record()
    for _ in range(n_dec):
        fused_recurrent_gated_delta_rule_step(dq, dk, dv, dg, db, state, out=do_buf)
    e3.record()
    barrier(world)
    return max_over_ranks(s3.elapsed_time(e3) / n_dec, world), dec_bytes


def long_prefill_bench(dev, rank, world, reps=3):
    """Config 4: one sequence of T = 262,144 tokens (H=16, d=128, bf16, forward only, in-kernel L2 norm),
    cut into `world` contiguous segments, one per rank (strong scaling: the sequence is fixed), each run as
    8 local pieces side by side (16 heads alone would fill 16 of 148 SMs): one prep pass, the pieces' C and
    M state passes, the scan of the affine maps with one NCCL all_gather of every rank's map, and the
    outputs pass from every piece's true incoming state. Returns ms per call, max over ranks."""
    import torch

    from sorernn_b200.seqsplit import segmented_prefill

    T, H, D, P = 262144, 16, 128, 8
    Tr = T // world
    x = make_inputs(1, Tr, H, D, dev, seed=4000 + rank)

    def call():
        with torch.no_grad():
            segmented_prefill(x["q"], x["k"], x["v"], x["g"], x["beta"], use_qk_l2norm_in_kernel=True,
                              local_segments=P)

    call()
    barrier(world)
    s0, e0 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record()
    for _ in range(reps):
        call()
    e0.record()
    barrier(world)
    ms = max_over_ranks(s0.elapsed_time(e0) / reps, world)
    return {"config": f"config4: B1 T{T} H{H} d{D} bf16 forward, {world} rank segment(s) x {P} local pieces",
            "ms_per_call": round(ms, 3), "tokens_per_s": round(T / (ms / 1e3), 1), "reps": reps,
            "useful_tflops": round(T * H * FWD_FLOP_PER_TOKEN_HEAD / (ms / 1e3) / 1e12, 2)}


def layer_ops_bench(dev, world, hbm_peak, reps=10):
    """The layer's neighbouring steps at config-1 sizes (B=8, T=4096, H=16, d=128, bf16): the output step
    RMSNorm(o)*silu(gate) over o [8, 4096, 16, 128] and the q-projection's causal conv + SiLU over
    [8, 4096, 2048] (K = 4), forward and backward through the public ops (torch.autograd.grad, so no
    gradient accumulation kernels run), one call captured as a CUDA graph and replayed. HBM-bound: reports
    GB/s of the algorithmic bytes (each tensor read or written once) per call and its fraction of the
    measured HBM peak, max over ranks."""
    import torch

    from sorernn_b200.layer_ops import causal_conv1d, rms_norm_gated

    gen = torch.Generator(device=dev).manual_seed(7)
    B, T, H, D = CFG1["B"], CFG1["T"], CFG1["H"], CFG1["D"]
    o = torch.randn(B, T, H, D, device=dev, generator=gen).bfloat16().requires_grad_(True)
    gate = torch.randn(B, T, H, D, device=dev, generator=gen).bfloat16().requires_grad_(True)
    w = torch.ones(D, device=dev, requires_grad=True)
    dy = torch.randn(B, T, H, D, device=dev, generator=gen).bfloat16()
    xc = torch.randn(B, T, H * D, device=dev, generator=gen).bfloat16().requires_grad_(True)
    wc = (torch.randn(H * D, 4, device=dev, generator=gen) * 0.5).requires_grad_(True)
    dyc = torch.randn(B, T, H * D, device=dev, generator=gen).bfloat16()
    nb = o.numel() * 2  # bytes of one bf16 tensor of this size

    def timed(fn):
        # one fwd+bwd call captured as a CUDA graph and replayed: device time of the kernels, without the
        # per-call host dispatch of the Python autograd path (which a short op like these can be bound by)
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(2):
                fn()
        torch.cuda.current_stream(dev).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            fn()
        graph.replay()
        barrier(world)
        s0, e0 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        for _ in range(reps):
            graph.replay()
        e0.record()
        barrier(world)
        del graph
        return max_over_ranks(s0.elapsed_time(e0) / reps, world)

    def ng():
        y = rms_norm_gated(o, gate, w, None, activation="swish", eps=1e-6)
        torch.autograd.grad(y, (o, gate, w), dy)

    def cv():
        y = causal_conv1d(xc, wc, activation="silu")[0]
        torch.autograd.grad(y, (xc, wc), dyc)

    ms_ng, ms_cv = timed(ng), timed(cv)
    # fwd reads x, gate and writes y; bwd reads x, gate, dy and writes dx, dgate: 8 tensor passes
    # conv: fwd reads x, writes y; bwd reads x, dy, writes dx: 5 tensor passes
    gbs_ng, gbs_cv = 8 * nb / (ms_ng / 1e3) / 1e9, 5 * nb / (ms_cv / 1e3) / 1e9
    return {"config": "config1 sizes, bf16: rms_norm_gated over [8,4096,16,128]; causal_conv1d K=4 over [8,4096,2048]",
            "rms_norm_gated_fwd_bwd_ms": round(ms_ng, 4), "rms_norm_gated_gbs": round(gbs_ng, 1),
            "rms_norm_gated_hbm_frac": round(gbs_ng / hbm_peak, 4),
            "causal_conv1d_fwd_bwd_ms": round(ms_cv, 4), "causal_conv1d_gbs": round(gbs_cv, 1),
            "causal_conv1d_hbm_frac": round(gbs_cv / hbm_peak, 4)}


def activation_memory(leaf, do, step, zero):
    """Device memory of one config-1 fwd+bwd in each backward mode, from the caching allocator's counters:
    the bytes the forward leaves allocated until the backward (its output o, the final state and the op's
    own saved tensors; q, k, v, g, beta are the caller's and not counted) and the backward's peak above
    that (its transient workspace plus the gradients). Modes: the default (every chunk's backward record
    saved, the backward runs the reverse sweep alone) and the recompute mode (fp32 state checkpoints every
    8 chunks, the backward rebuilds the records first). Beside them, what storing every chunk's fp32 state
    would take (FLA's chunk_fwd_h materialises [B, NT, H, 128, 128] in its backward)."""
    import torch

    from sorernn_b200.gated_delta_rule import DEFAULT_CKPT_EVERY, SAVE_RECORDS, chunk_gated_delta_rule

    def one(ckpt_every):
        zero()
        torch.cuda.synchronize()
        base = torch.cuda.memory_allocated()
        o, _ = chunk_gated_delta_rule(leaf["q"], leaf["k"], leaf["v"], leaf["g"], leaf["beta"],
                                      use_qk_l2norm_in_kernel=True, ckpt_every=ckpt_every)
        torch.cuda.synchronize()
        held = torch.cuda.memory_allocated() - base
        o_bytes = o.numel() * o.element_size()
        torch.cuda.reset_peak_memory_stats()
        after_fwd = torch.cuda.memory_allocated()
        o.backward(do)
        torch.cuda.synchronize()
        bwd_peak = torch.cuda.max_memory_allocated() - after_fwd
        grads = sum(t.grad.numel() * t.grad.element_size() for t in leaf.values())
        del o
        zero()
        return {"held_fwd_to_bwd_bytes": held, "of_which_output_o": o_bytes, "op_saved_bytes": held - o_bytes,
                "bwd_peak_above_fwd_bytes": bwd_peak, "of_which_gradients": grads,
                "bwd_transient_bytes": bwd_peak - grads}

    B, T, H, D = leaf["q"].shape
    per_chunk_states = B * H * ((T + 63) // 64) * D * D * 4
    saved, recompute = one(SAVE_RECORDS), one(DEFAULT_CKPT_EVERY)
    recompute["ckpt_every_chunks"] = DEFAULT_CKPT_EVERY
    return {"saved_records (default)": saved, "recompute": recompute,
            "per_chunk_fp32_states_bytes": per_chunk_states,
            "recompute_saves_vs_per_chunk_states_bytes": per_chunk_states - recompute["op_saved_bytes"],
            "note": "torch.cuda.memory_allocated / max_memory_allocated around one call"}


def config2_layer_bench(dev, world, reps=5):
    """Config 2's GDN mixer layer (d_model 1536, 16 q/k heads and 16 v heads of 128, short conv K = 4,
    gate and beta activations in kernel, fused RMSNorm(o)*silu(gate)) through sorernn_b200.layer, fwd+bwd
    under bf16 autocast at batch 8 x 4096 (packed as one 32,768-token micro-batch of 8 documents, as the
    reference's trainer and bench pack, scripts/bench.py:84-111). The model's other layers (6 attention
    layers, SwiGLU FFNs, embeddings, MTP head) belong to the reference and are not built here; 18 of its
    24 layers are this one. Returns ms per layer call, tokens/s and the peak device memory of one call."""
    import torch

    from sorernn_b200.layer import GatedDeltaNet

    B, T, d = 8, 4096, 1536
    gen = torch.Generator(device=dev).manual_seed(9)
    torch.manual_seed(9)
    layer = GatedDeltaNet(d, 16, 16, 128).to(dev)
    x = (torch.randn(1, B * T, d, device=dev, generator=gen) * 0.5).requires_grad_(True)
    dy = torch.randn(1, B * T, d, device=dev, generator=gen)
    cu_cpu = torch.arange(0, B * T + 1, T, dtype=torch.int64)
    cu = cu_cpu.to(dev)

    def call():
        x.grad = None
        layer.zero_grad(set_to_none=True)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            y = layer(x, cu_seqlens=cu, cu_seqlens_cpu=cu_cpu)
        y.backward(dy)

    call()
    barrier(world)
    torch.cuda.reset_peak_memory_stats(dev)
    base = torch.cuda.memory_allocated(dev)
    s0, e0 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record()
    for _ in range(reps):
        call()
    e0.record()
    barrier(world)
    ms = max_over_ranks(s0.elapsed_time(e0) / reps, world)
    peak = torch.cuda.max_memory_allocated(dev) - base
    return {"workload": "config2 GDN layer: d_model 1536, 16+16 heads x 128, conv 4, gate in kernel, fused "
                        "norm-gate, 8 documents x 4096 packed, bf16 autocast, fwd+bwd",
            "ms_per_layer": round(ms, 3), "tokens_per_s_per_layer": round(B * T / (ms / 1e3), 1),
            "gdn_layers_in_model": 18, "ms_gdn_share_of_step": round(18 * ms, 2),
            "peak_bytes_per_call": int(peak),
            "not_built": "attention, FFN, embedding and MTP layers of SoreLM (reference code, out of scope)"}


def strong_scaling_bench(dev, rank, world, steps):
    """Config 1 with its total work fixed: the B=8 rows (x 16 heads) are split across the ranks (B/N rows
    per rank, i.e. 128/N (sequence, head) units) and every rank times fwd+bwd of its share; value = the
    8 x 4096 tokens / the slowest rank's time per step (strong scaling). The main line is the weak one
    (every rank a full B=8 problem). With fewer than 128 units per rank the rank's sequences are also run
    cut into P = 128 / units pieces side by side (sorernn_b200.pieces, no collective); both paths are timed
    and the line reports each and the faster."""
    import torch

    from sorernn_b200 import chunk_gated_delta_rule
    from sorernn_b200.pieces import chunk_gated_delta_rule_pieces

    B, T, H, D = CFG1["B"], CFG1["T"], CFG1["H"], CFG1["D"]
    if B % world:
        return {"skipped": f"B={B} rows do not split over {world} ranks"}
    Br = B // world
    units = Br * H
    x = make_inputs(Br, T, H, D, dev, seed=77 + rank)
    leaf = {n: x[n].clone().requires_grad_(n != "do") for n in ("q", "k", "v", "g", "beta")}
    P = 1
    while units * P * 2 <= 128 and T % (64 * P * 2) == 0:
        P *= 2

    def step(inp, do):  # the sequences whole (the op would otherwise pick pieces by itself below 33 units)
        o, _ = chunk_gated_delta_rule(inp["q"], inp["k"], inp["v"], inp["g"], inp["beta"], use_qk_l2norm_in_kernel=True,
                                      pieces=1)
        o.backward(do)

    def pieces_step_of(Pn):
        def pieces_step(inp, do):
            o, _ = chunk_gated_delta_rule_pieces(inp["q"], inp["k"], inp["v"], inp["g"], inp["beta"], pieces=Pn,
                                                 use_qk_l2norm_in_kernel=True)
            o.backward(do)
        return pieces_step

    def zero_s():
        for t in leaf.values():
            t.grad = None

    def timed(fn):
        for _ in range(3):
            zero_s()
            fn(leaf, x["do"])
        barrier(world)
        s0, e0 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        for _ in range(steps):
            zero_s()
            fn(leaf, x["do"])
        e0.record()
        barrier(world)
        return max_over_ranks(s0.elapsed_time(e0) / steps, world)

    ms_plain = timed(step)
    ms_pieces = None
    if P > 1:  # the largest piece count that keeps the CTAs within one wave, and half of it
        tried = {Pn: timed(pieces_step_of(Pn)) for Pn in sorted({P, max(2, P // 2)})}
        P = min(tried, key=tried.get)
        ms_pieces = tried[P]
    ms = ms_plain if ms_pieces is None else min(ms_plain, ms_pieces)
    out = {"workload": f"config1 B{B} T{T} H{H} d{D} fwd+bwd split by batch rows over {world} rank(s)",
           "per_rank_batch": Br, "units_per_rank": units, "ms_per_step": round(ms, 4),
           "tokens_per_s": round(B * T / (ms / 1e3), 1), "scaling": "strong",
           "ms_per_step_one_piece": round(ms_plain, 4)}
    if ms_pieces is not None:
        out.update({"pieces_per_sequence": P, "ms_per_step_pieces": round(ms_pieces, 4),
                    "pieces_tried_ms": {str(k): round(v, 4) for k, v in tried.items()},
                    "path": "pieces" if ms_pieces < ms_plain else "one piece"})
    out["limiter"] = STRONG_LIMITER.format(units=units) if P == 1 else STRONG_LIMITER_PIECES.format(
        units=units, P=P, chunks=T // (64 * P))
    return out


def run_ours(args):
    import torch

    from sorernn_b200 import _lib
    from sorernn_b200 import chunk_gated_delta_rule

    rank, world, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    if args.profile_layer:  # profiling mode: the layer-neighbour ops only, two fwd+bwd calls each (no JSON line)
        layer_ops_bench(dev, world, 1.0, reps=1)
        print(json.dumps({"profile_layer": True, "ok": True}))
        return
    if args.profile_decode:  # profiling mode: decode steps only (no JSON line)
        decode_bench(dev, rank, world, n_dec=args.profile_decode, timed=False)
        print(json.dumps({"profile_decode": args.profile_decode, "ok": True}))
        return
    B, T, H, D = CFG1["B"], CFG1["T"], CFG1["H"], CFG1["D"]
    if args.profile_batch:
        B = args.profile_batch  # profiling mode: a small case, fwd+bwd steps only (no JSON line)
    x = make_inputs(B, T, H, D, dev, seed=1234 + rank)
    leaf = {n: x[n].clone().requires_grad_(n != "do") for n in ("q", "k", "v", "g", "beta")}
    # profiling mode runs whole sequences unless --profile-pieces asks for pieces (at batch 1 or 2 the op would
    # otherwise pick pieces by itself); the timed run (batch 8, 128 sequence-heads) never splits
    pieces = args.profile_pieces if args.profile_batch else None

    def step(inp, do, ev=None):
        if ev is not None:
            ev[0].record()
        o, _ = chunk_gated_delta_rule(inp["q"], inp["k"], inp["v"], inp["g"], inp["beta"],
                                      use_qk_l2norm_in_kernel=True, pieces=pieces)
        if ev is not None:
            ev[1].record()
        o.backward(do)
        if ev is not None:
            ev[2].record()
        return o

    def zero():
        for t in leaf.values():
            t.grad = None

    for _ in range(args.warmup):
        zero()
        step(leaf, x["do"])
    barrier(world)
    mem = activation_memory(leaf, x["do"], step, zero) if not args.profile_batch else None
    if args.profile_batch:
        for _ in range(args.steps):
            zero()
            step(leaf, x["do"])
        torch.cuda.synchronize()
        print(json.dumps({"profile_batch": B, "steps": args.steps, "ok": True}))
        return
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = _lib.lib().gdn_kernel_launches()
    with ClockSampler(local) as clk:
        barrier(world)
        start.record()
        for i in range(args.steps):
            zero()
            step(leaf, x["do"], evs[i])
        end.record()
        barrier(world)
    launches = _lib.lib().gdn_kernel_launches() - launches0
    ms_local = start.elapsed_time(end) / args.steps
    ms = max_over_ranks(ms_local, world)
    fwd_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in evs)
    bwd_ms = statistics.mean(e[1].elapsed_time(e[2]) for e in evs)
    tokens = B * T * world
    value = tokens / (ms / 1e3)

    # e2e through the public API from pinned host memory
    host = {n: t.detach().cpu().pin_memory() for n, t in x.items()}
    outs = {n: torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for n, t in x.items() if n != "do"}
    o_host = torch.empty(x["v"].shape, dtype=x["v"].dtype, pin_memory=True)
    h2d = sum(t.numel() * t.element_size() for t in host.values())
    d2h = o_host.numel() * o_host.element_size() + sum(t.numel() * t.element_size() for t in outs.values())

    # Pipelined like a training input loader: step i+1's inputs cross PCIe (copy_in stream) while step i
    # computes, and step i's output and gradients come back (copy_out stream) while step i+1 computes.
    # Every step's inputs are copied from pinned host memory and its results read back inside the timed
    # region; device input buffers are double-buffered.
    compute = torch.cuda.current_stream(dev)
    copy_in, copy_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    dbuf = [{n: torch.empty_like(x[n]) for n in host} for _ in range(2)]
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_free = [torch.cuda.Event() for _ in range(2)]

    def e2e_run(n_steps):
        copy_in.wait_stream(compute)
        for i in range(n_steps + 1):
            if i < n_steps:  # inputs of step i (slot i % 2 is free once step i-2's compute finished)
                slot = i % 2
                with torch.cuda.stream(copy_in):
                    if i >= 2:
                        copy_in.wait_event(ev_free[slot])
                    for n in host:
                        dbuf[slot][n].copy_(host[n], non_blocking=True)
                    ev_in[slot].record(copy_in)
            if i >= 1:  # compute step i-1, then queue its results' read-back
                j, slot = i - 1, (i - 1) % 2
                compute.wait_event(ev_in[slot])
                inp = {n: dbuf[slot][n].detach().requires_grad_(n != "do") for n in host}
                o = step(inp, inp["do"])
                ev_free[slot].record(compute)
                copy_out.wait_stream(compute)
                with torch.cuda.stream(copy_out):
                    o_host.copy_(o.detach(), non_blocking=True)
                    o.record_stream(copy_out)
                    for n in outs:
                        outs[n].copy_(inp[n].grad, non_blocking=True)
                        inp[n].grad.record_stream(copy_out)
        compute.wait_stream(copy_out)

    e2e_run(2)
    e2e_steps = max(3, min(4 * args.steps, 32))  # the pipeline fill and drain (one copy each way) amortised
    torch.cuda.synchronize(dev)
    barrier(world)
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s2.record(compute)
    e2e_run(e2e_steps)
    e2.record(compute)
    torch.cuda.synchronize(dev)
    barrier(world)
    e2e_ms = max_over_ranks(s2.elapsed_time(e2) / e2e_steps, world)

    strong = strong_scaling_bench(dev, rank, world, args.steps)
    config2 = config2_layer_bench(dev, world)
    dec_ms, dec_bytes = decode_bench(dev, rank, world)
    long_prefill = long_prefill_bench(dev, rank, world)
    peaks, peak_kind = load_peaks()
    layer_ops = layer_ops_bench(dev, world, peaks["hbm_gbs"])
    layer_ops["peak_source"] = f"{peak_kind} hbm_gbs (of {peak_kind})"
    dec_gbs = dec_bytes / (dec_ms / 1e3) / 1e9

    # roofline of the dominant kernel (the backward launch): algorithmic flops / measured duration
    bwd_flop = 2 * FWD_FLOP_PER_TOKEN_HEAD * B * T * H
    fwd_flop = FWD_FLOP_PER_TOKEN_HEAD * B * T * H
    peak_tf = peaks["bf16_tflops"]  # burst: the timed region is tens of ms, not a seconds-long loop
    achieved_bwd = bwd_flop / (bwd_ms / 1e3) / 1e12
    rec = {
        "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded; config-0 value distributions)",
        "config": {"workload": "config1: GDN op fwd+bwd B8 T4096 H16 dk=dv=128 bf16, fp32 g/state, chunk 64, "
                               "in-kernel qk L2 norm", "per_rank_batch": B, "seq_len": T, "heads": H,
                   "parallelism": f"batch x head shards, dp{world}",
                   "l2": "inputs (~0.8 GB/rank) exceed the 126 MB L2; no flush"},
        "e2e": {"value": round(tokens / (e2e_ms / 1e3), 1), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 3), "steps": e2e_steps,
                "overlap": "pinned-host copies on two side streams: step i+1's inputs in and step i's "
                           "results out while step i computes"},
        "gpu_launches": int(launches),
        "kernels": {"fwd_ms": round(fwd_ms, 4), "bwd_ms": round(bwd_ms, 4),
                    "fwd_tflops": round(fwd_flop / (fwd_ms / 1e3) / 1e12, 2)},
        "roofline": {"bound": "tensor", "kernel": "backward pass (reverse-sweep launch over the saved records)",
                     "achieved": round(achieved_bwd, 2), "peak": peak_tf, "unit": "TFLOP/s",
                     "frac": round(achieved_bwd / peak_tf, 4),
                     "peak_source": f"{peak_kind} bf16_tflops, the burst figure (of {peak_kind})",
                     "traffic": BWD_PASS_TRAFFIC_BYTES * B / 8,
                     "traffic_note": "ncu DRAM read+write bytes per call, batch-2 capture scaled"},
        "decode": {"metric": "decode-step HBM GB/s (config 3: 256 seq x H16 x 128x128 fp32 state per GPU)",
                   "value": round(dec_gbs * world, 1), "unit": "GB/s (all GPUs)", "per_gpu_gbs": round(dec_gbs, 1),
                   "us_per_step": round(dec_ms * 1e3, 2),
                   "roofline": {"bound": "hbm", "achieved": round(dec_gbs, 1), "peak": peaks["hbm_gbs"],
                                "unit": "GB/s", "frac": round(dec_gbs / peaks["hbm_gbs"], 4),
                                "peak_source": f"{peak_kind} hbm_gbs (of {peak_kind})",
                                "traffic": DECODE_TRAFFIC_BYTES, "algorithmic_bytes": dec_bytes}},
        "clocks": clk.summary(),
        "long_prefill": long_prefill,
        "layer_ops": layer_ops,
        "activation_memory": mem,
        "config1_strong": strong,
        "config2_gdn_layer": config2,
    }
    if rank == 0:
        if world == 1:  # the host-core baseline is timed at N=1 only
            rec["cpu_baseline"] = cpu_baseline(seconds=args.cpu_seconds)
        print(json.dumps(rec), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()


def cpu_baseline(seconds=15.0, threads=0):
    """The reference recurrence (C restatement in oracle/, fwd + bwd) on the host cores, on a bounded
    sample of config 1: one batch row (T=4096, H=16) truncated to the tokens that fit the time budget."""
    import numpy as np

    from oracle import cgdn

    threads = threads or os.cpu_count() or 1
    H, D, T = CFG1["H"], CFG1["D"], CFG1["T"]
    B, T_s = 1, 512
    while True:
        rng = np.random.default_rng(5)
        q = rng.standard_normal((B, T_s, H, D)).astype(np.float32)
        k = rng.standard_normal((B, T_s, H, D)).astype(np.float32)
        v = rng.standard_normal((B, T_s, H, D)).astype(np.float32)
        g = (-np.logaddexp(0, -rng.standard_normal((B, T_s, H))) / 16).astype(np.float32)
        beta = (1 / (1 + np.exp(-rng.standard_normal((B, T_s, H))))).astype(np.float32)
        do = rng.standard_normal((B, T_s, H, D)).astype(np.float32)
        t0 = time.perf_counter()
        cgdn.forward(q, k, v, g, beta, D ** -0.5, use_qk_l2norm=True, threads=threads)
        cgdn.backward(q, k, v, g, beta, do, D ** -0.5, use_qk_l2norm=True, threads=threads)
        dt = time.perf_counter() - t0
        if dt * 2.2 > seconds or (B >= CFG1["B"] and T_s >= T):
            break
        if T_s < T:
            T_s *= 2
        else:
            B *= 2
    return {"value": round(B * T_s / dt, 2), "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"fwd+bwd of B={B} rows x T={T_s} tokens (config 1 is B=8 x T=4096), H=16, d=128, fp32, "
                      f"{dt:.2f} s"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import numpy as np  # noqa: F401

    vals = []
    for _ in range(args.warmup):
        cpu_baseline(seconds=args.cpu_seconds / 4)
    for _ in range(args.steps):
        vals.append(cpu_baseline(seconds=args.cpu_seconds / 4))
    v = statistics.median(x["value"] for x in vals)
    cb = dict(vals[-1])
    cb["value"] = v
    # ms_per_step: one config-1 step (B x T tokens) at the sampled rate
    rec = {"impl": "reference", "metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": args.gpus,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(CFG1["B"] * CFG1["T"] / v * 1e3, 1),
           "higher_is_better": True, "scaling": "weak",
           "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)",
           "config": {"workload": "config1 on host cores: reference recurrence fwd+bwd (C port of "
                                  "sore/model/gdn_ref.py) of B8 T4096 H16 d128 rows, each step a bounded "
                                  "sample of them (see cpu_baseline.sample)"},
           "cpu_baseline": cb, "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                                       "d2h_bytes_per_step": 0}}
    print(json.dumps(rec), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--profile-batch", type=int, default=0,
                    help="profiling mode: run only fwd+bwd steps of config 1 with this batch (for ncu captures)")
    ap.add_argument("--profile-pieces", type=int, default=1,
                    help="with --profile-batch: pieces per sequence (1: whole sequences)")
    ap.add_argument("--profile-decode", type=int, default=0,
                    help="profiling mode: run only this many decode steps of config 3 (for ncu captures)")
    ap.add_argument("--profile-layer", action="store_true",
                    help="profiling mode: run only the layer-neighbour ops at config-1 sizes (for ncu captures)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
