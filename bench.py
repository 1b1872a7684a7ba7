#!/usr/bin/env python
"""Benchmark of the paged-decode hot path on B200.

Workload (default): Llama-3-8B attention shape, FP16, 32 query / 8 KV heads,
head_dim 128, 32 layers, block 16, batch 256, lengths lognormal(median 1024,
sigma 0.8) clipped to [16, 8192], RoPE theta 5e5, fragmented block tables,
sequences sharded evenly over the ranks (each rank owns its pools/tables).

One step = one decode token for every sequence through all 32 layers'
attention ops: rope_kv_write (RoPE + paged KV-slot write) then paged_attention.
Metric: seq-steps/s (sequences advanced one token through all layers per
second), whole job. Inputs (60 GB of KV pools at batch 256) are far larger
than L2, so no flush is needed between steps.

  python bench.py [--gpus N --steps K --warmup W] [--impl ours|reference]
  torchrun --nproc-per-node N bench.py --gpus N ...   (one rank per GPU)

Second workload, ``--workload smollm_tick``: one decode tick of a random-init
SmolLM2-135M architecture (FP16, 30 layers, 9/3 heads, head_dim 64) for 128
sequences with lengths U[16, 4096] on pages reused in arbitrary order; the
whole model runs (embedding, projections, MLP, LM head in PyTorch/cuBLAS;
RoPE, KV writes, metadata and attention on this library), one replica per
GPU. Ours: llama_runner.PagedLlama with graph-captured ticks. Reference arm:
the reference's PagedLlama.decode (restated in oracle/llama_model.py, pinned
to its logits) with the reference's own CUDA attention kernel when it was
built into oracle/_ref, else its torch path.

Fourth workload, ``--workload prefill_write``: the prefill RoPE + paged KV
write of the same 16 prompts (worker/llama.py:128-140), one layer per step.

Third workload, ``--workload prefill``: the prefill attention of 16 prompts
with lengths U[64, 1024] (SmolLM2 heads 9/3, head_dim 64, FP16), one layer
per step. Ours: prefill_attention over the paged pools. Reference arm: the
reference's prefill attention (worker/llama.py:141-144: repeat_interleave
of K/V and causal SDPA over the padded batch) on the same GPU.

Prints one JSON line (rank 0).
"""
from __future__ import annotations

import argparse
import importlib
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))
PKG = importlib.import_module("distributed-llm-inference_b200")
W = importlib.import_module("distributed-llm-inference_b200.workloads")

METRIC = "paged-attn decode seq-steps/s"
UNIT = "seq-steps/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["llama3_8b", "smollm_fp16", "smollm_fp32",
                                           "smollm_tick", "prefill", "prefill_write"],
                    default="llama3_8b")
    ap.add_argument("--batch", type=int, default=None, help="override the workload batch")
    ap.add_argument("--layers", type=int, default=None, help="override the layer count (profiling)")
    ap.add_argument("--sharding", choices=["balanced", "contiguous"], default="balanced",
                    help="how sequences are split over ranks (both give every rank B/P)")
    ap.add_argument("--no-alt", action="store_true",
                    help="at N>1, skip the second measurement with the other sharding")
    ap.add_argument("--prefill-kernel", choices=["auto", "tcgen05", "mma"], default="auto",
                    help="pin the prefill attention kernel (prefill workload)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-secondary", action="store_true",
                    help="skip the other configurations' measurements (the `secondary` object)")
    return ap.parse_args()


def make_workload(args):
    if args.workload == "llama3_8b":
        return W.llama3_8b(batch=args.batch or 256, layers=args.layers or 32)
    if args.workload == "smollm_fp32":
        return W.smollm_fp32(batch=args.batch or 64, layers=args.layers or 30)
    return W.smollm_fp16(batch=args.batch or 64, layers=args.layers or 30)


def decode_config(full, args, world: int) -> dict:
    """The headline line's config, identical in both arms: the workload, the
    sharding of its sequences over `world` ranks and the L2 note."""
    ranks = [full.shard(r, world, args.sharding) for r in range(world)] if world > 1 else [full]
    w0 = ranks[0]
    return {
        "workload": (f"{full.name}: batch {full.batch}, {full.heads}/{full.kv_heads} heads, "
                     f"head_dim {full.head_dim}, {full.layers} layers, block {full.block_size}, "
                     "lengths lognormal(1024, 0.8) in [16, 8192]"
                     if args.workload == "llama3_8b" else full.name),
        "batch": full.batch, "layers": full.layers, "max_length": full.max_length,
        "mean_length": float(full.lengths.float().mean()),
        "sharding": (f"{args.sharding}: every rank owns B/P whole sequences and its own "
                     "pools/tables" + ("; balanced = dealt longest-first to the rank with "
                                       "the fewest KV tokens" if args.sharding == "balanced"
                                       else "; contiguous = sequences [r*B/P, (r+1)*B/P)")),
        "max_rank_tokens": max(float(r.lengths.sum()) for r in ranks),
        "mean_rank_tokens": float(full.lengths.sum()) / world,
        "l2": "inputs larger than L2 (KV pools %.1f GB per rank)" % (
            2 * w0.layers * w0.num_blocks * w0.block_size * w0.kv_heads * w0.head_dim
            * w0.elem_bytes / 1e9),
    }


# --------------------------------------------------------------------------
# clocks sampled during the timed region (NVML; reading only)
# --------------------------------------------------------------------------
REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
           0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
           0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
           0x100: "display_clock_setting"}


class ClockSampler:
    def __init__(self, device_index: int, period_s: float = 0.02):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self.period = period_s
        self._stop = threading.Event()
        self._thread = None
        self.error = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nvml = pynvml
            self._h = self._handle(pynvml, torch.cuda.get_device_properties(device_index))
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception as e:  # noqa: BLE001 - report, never fail the bench
            self.error = f"nvml unavailable: {e}"
            self._nvml = None

    @staticmethod
    def _handle(nv, props):
        """NVML handle of the CUDA device: match by UUID, else by the PCI
        address string built from torch's integer domain/bus/device ids."""
        want = str(props.uuid).lower().removeprefix("gpu-")
        for i in range(nv.nvmlDeviceGetCount()):
            h = nv.nvmlDeviceGetHandleByIndex(i)
            uid = nv.nvmlDeviceGetUUID(h)
            uid = (uid.decode() if isinstance(uid, bytes) else str(uid)).lower().removeprefix("gpu-")
            if uid == want:
                return h
        addr = "%08X:%02X:%02X.0" % (int(props.pci_domain_id), int(props.pci_bus_id),
                                     int(props.pci_device_id))
        return nv.nvmlDeviceGetHandleByPciBusId(addr.encode())

    def _run(self):
        nv = self._nvml
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                for bit, name in REASONS.items():
                    if r & bit and bit != 0x1:
                        self.reasons.add(name)
            except Exception as e:  # noqa: BLE001
                self.error = str(e)
            time.sleep(self.period)

    def start(self):
        if self._nvml is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()

    def stop(self) -> dict:
        if self._thread is not None:
            self._stop.set()
            self._thread.join()
        out = {"sm_mhz": statistics.median(self.samples) if self.samples else None,
               "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
               "samples": len(self.samples)}
        if self.error:
            out["note"] = self.error
        return out


# --------------------------------------------------------------------------
# distributed plumbing
# --------------------------------------------------------------------------
def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def max_over_ranks(x: float, world: int, device) -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int, device):
    if world > 1:
        import torch.distributed as dist
        dist.barrier(device_ids=[device.index])


# --------------------------------------------------------------------------
# our arm
# --------------------------------------------------------------------------
class DecodeStep:
    """All layers of one decode step through the public ops, with
    preallocated outputs so the step can be captured in a CUDA graph."""

    def __init__(self, w, t, fused=True):
        self.w, self.t = w, t
        self.q_out = [torch.empty_like(q) for q in t.q]
        self.k_out = [torch.empty_like(k) for k in t.k]
        self.out = [torch.empty_like(q) for q in t.q]
        # one launch per layer (decode_attention) where the fused kernel applies
        self.fused = fused and PKG.decode_attention_supported(t.q[0], t.k_pools[0])

    def layer(self, layer):
        """RoPE + KV-slot write + attention of one layer (one or two launches)."""
        t = self.t
        if self.fused:
            PKG.decode_attention(t.q[layer], t.k[layer], t.v[layer], t.k_pools[layer],
                                 t.v_pools[layer], t.tables, t.lengths, t.inv_freq,
                                 self.w.max_length, out=self.out[layer],
                                 metadata_stable=layer > 0, pools_stable=layer > 0)
        else:
            self.prologue(layer)
            self.attention(layer)

    def prologue(self, layer):
        t = self.t
        PKG.rope_kv_write(t.q[layer], t.k[layer], t.v[layer], t.k_pools[layer], t.v_pools[layer],
                          t.physical, t.offsets, t.positions, t.inv_freq,
                          q_out=self.q_out[layer], k_out=self.k_out[layer])

    def attention(self, layer):
        t = self.t
        PKG.paged_attention(self.q_out[layer], t.k_pools[layer], t.v_pools[layer], t.tables,
                            t.lengths, self.w.max_length, out=self.out[layer])

    def __call__(self):
        for layer in range(self.w.layers):
            self.layer(layer)


def capture(fn, stream):
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        fn()
    return g


def time_graph(g, reps, stream):
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        s.record(stream)
        for _ in range(reps):
            g.replay()
        e.record(stream)
    e.synchronize()
    return s.elapsed_time(e)


def e2e_run(w, t, steps, warmup, device):
    """Public-API path with host buffers: every step copies each layer's new
    q/k/v (and the step's metadata: tables and lengths, plus positions and
    slots for the two-launch path) from pinned host memory, runs
    decode_attention (or rope_kv_write + paged_attention where the fused
    kernel does not apply), and copies each layer's attention output back to
    pinned host memory. Layers move in groups: a group's inputs sit side by
    side in one pinned buffer and arrive with one copy, while the previous
    group computes; its outputs leave with one copy while the next group
    computes (separate copy streams, event ordering). The first and the last
    group hold one layer, so little copy time is left outside the compute."""
    L = w.layers
    fused = PKG.decode_attention_supported(t.q[0], t.k_pools[0])
    meta = (t.tables, t.lengths) if fused else (t.tables, t.lengths, t.positions, t.physical,
                                                t.offsets)

    def packed(tensors, pin):
        """One buffer holding `tensors` back to back (each part 16-byte
        aligned), and a view of it shaped like each tensor."""
        sizes = [x.numel() * x.element_size() for x in tensors]
        offs, total = [], 0
        for n in sizes:
            offs.append(total)
            total += (n + 15) // 16 * 16
        buf = (torch.empty(total, dtype=torch.uint8, pin_memory=True) if pin
               else torch.empty(total, dtype=torch.uint8, device=device))
        views = [buf[o:o + n].view(x.dtype).view(x.shape) for x, o, n in zip(tensors, offs, sizes)]
        return buf, views

    inner = 4
    sizes = [1] + [inner] * ((L - 2) // inner) + ([(L - 2) % inner] if (L - 2) % inner else [])
    sizes = (sizes + [1]) if L > 1 else [1]
    groups, first = [], 0
    for n in sizes:
        groups.append(list(range(first, first + n)))
        first += n
    assert first == L
    # inputs: per group [q, k, v of each layer]; outputs: per group [out of each layer]
    h_in, d_in, h_outb, d_outb = [], [], [], []
    d_q, d_k, d_v, d_out, h_out = [None] * L, [None] * L, [None] * L, [None] * L, [None] * L
    for grp in groups:
        parts = [x for layer in grp for x in (t.q[layer], t.k[layer], t.v[layer])]
        hb, hv = packed(parts, True)
        db, dv = packed(parts, False)
        for i, layer in enumerate(grp):
            for j in range(3):
                hv[3 * i + j].copy_(parts[3 * i + j])
            d_q[layer], d_k[layer], d_v[layer] = dv[3 * i], dv[3 * i + 1], dv[3 * i + 2]
        h_in.append(hb)
        d_in.append(db)
        outs = [t.q[layer] for layer in grp]
        ob, ov = packed(outs, True)
        dob, dov = packed(outs, False)
        for i, layer in enumerate(grp):
            h_out[layer], d_out[layer] = ov[i], dov[i]
        h_outb.append(ob)
        d_outb.append(dob)
    h_meta_b, h_meta = packed(list(meta), True)
    for hm, x in zip(h_meta, meta):
        hm.copy_(x)
    d_meta_b, d_meta = packed(list(meta), False)
    q_out = [torch.empty_like(x) for x in t.q]
    k_out = [torch.empty_like(x) for x in t.k]
    comp = torch.cuda.Stream(device)
    h2d = torch.cuda.Stream(device)
    d2h = torch.cuda.Stream(device)
    copied = [torch.cuda.Event() for _ in range(len(groups) + 1)]
    done = [torch.cuda.Event() for _ in range(len(groups))]
    h2d_bytes = sum(x.numel() * x.element_size() for x in list(t.q) + list(t.k) + list(t.v)
                    + list(meta))
    d2h_bytes = sum(x.numel() * x.element_size() for x in t.q)

    def step():
        with torch.cuda.stream(h2d):
            h2d.wait_stream(comp)  # previous step's kernels no longer read the buffers
            d_meta_b.copy_(h_meta_b, non_blocking=True)
            copied[-1].record(h2d)
            for gi in range(len(groups)):
                d_in[gi].copy_(h_in[gi], non_blocking=True)
                copied[gi].record(h2d)
        comp.wait_event(copied[-1])
        tables, lengths = d_meta[0], d_meta[1]
        for gi, grp in enumerate(groups):
            comp.wait_event(copied[gi])
            for layer in grp:
                if fused:
                    PKG.decode_attention(d_q[layer], d_k[layer], d_v[layer], t.k_pools[layer],
                                         t.v_pools[layer], tables, lengths, t.inv_freq,
                                         w.max_length, out=d_out[layer],
                                         metadata_stable=layer > 0, pools_stable=layer > 0)
                else:
                    positions, physical, offsets = d_meta[2:]
                    PKG.rope_kv_write(d_q[layer], d_k[layer], d_v[layer], t.k_pools[layer],
                                      t.v_pools[layer], physical, offsets, positions, t.inv_freq,
                                      q_out=q_out[layer], k_out=k_out[layer])
                    PKG.paged_attention(q_out[layer], t.k_pools[layer], t.v_pools[layer],
                                        tables, lengths, w.max_length, out=d_out[layer])
            done[gi].record(comp)
            with torch.cuda.stream(d2h):
                d2h.wait_event(done[gi])
                h_outb[gi].copy_(d_outb[gi], non_blocking=True)
        comp.wait_stream(d2h)

    # The step (copies on their streams + ops) is captured as one CUDA graph,
    # as a serving loop would run it; eager launches if capture is refused.
    with torch.cuda.stream(comp):
        for _ in range(warmup):
            step()
        torch.cuda.synchronize(device)
        mode, run = "eager", step
        try:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=comp):
                step()
            torch.cuda.synchronize(device)
            mode, run = "graph", g.replay
            for _ in range(2):
                run()
            torch.cuda.synchronize(device)
        except Exception as err:  # noqa: BLE001 - fall back to eager launches
            print(f"e2e graph capture failed, timing eager launches: {err}", file=sys.stderr)
            torch.cuda.synchronize(device)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(comp)
        for _ in range(steps):
            run()
        e.record(comp)
    e.synchronize()
    ms = s.elapsed_time(e) / steps
    check = float(h_out[-1].float().abs().sum())  # the step's result, read on the host
    return ms, h2d_bytes, d2h_bytes, check, mode


def cpu_baseline(w, t, budget_s=15.0, sample=16):
    """The reference's CPU path (oracle port of worker/llama.py:108-117,
    :171-172, :58-71) on `sample` sequences of layer 0, all host threads,
    padded to the batch max_length like the reference; scaled to seq-steps/s
    over all layers."""
    sys.path.insert(0, str(REPO))
    from oracle import kv_cache, paged_attention as opa, rope as orope
    idx = torch.arange(min(sample, w.batch))
    tabs, (kp, vp) = W.compact_pages(w.tables[idx], w.lengths[idx], [t.k_pools[0], t.v_pools[0]],
                                     w.block_size)
    q = t.q[0][: len(idx)].cpu()
    k = t.k[0][: len(idx)].cpu()
    v = t.v[0][: len(idx)].cpu()
    lens = w.lengths[idx]
    pos = (lens.to(torch.int64) - 1).unsqueeze(1)
    phys = tabs.to(torch.int64).gather(1, (pos // w.block_size))[:, 0]
    off = pos[:, 0] % w.block_size
    inv = t.inv_freq.cpu()
    times = []
    t_end = time.perf_counter() + budget_s
    while time.perf_counter() < t_end or not times:
        t0 = time.perf_counter()
        qr, kr = orope.rope(q.unsqueeze(1), k.unsqueeze(1), pos, inv)
        kv_cache.write_decode(kp, phys, off, kr[:, 0])
        kv_cache.write_decode(vp, phys, off, v)
        opa.paged_attention(qr[:, 0], kp, vp, tabs, lens, w.max_length)
        times.append(time.perf_counter() - t0)
        if len(times) >= 3:
            break
    per_layer = statistics.median(times)
    return {"value": len(idx) / (per_layer * w.layers), "unit": UNIT,
            "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{len(idx)} of {w.batch} sequences x layer 0, scaled by {w.layers} layers "
                      f"(all layers have the same shapes); padded to max_length {w.max_length} "
                      f"like the reference; median of {len(times)} runs; os.cpu_count()={os.cpu_count()}"}


def run_ours(args):
    world, rank, local = dist_env()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=device)
    PKG.load_library()
    full = make_workload(args)
    w = full.shard(rank, world, args.sharding) if world > 1 else full
    t = W.materialize(w, device)
    step = DecodeStep(w, t)
    stream = torch.cuda.Stream(device)

    # warm caches (occupancy, workspace) on the capture stream, then capture
    with torch.cuda.stream(stream):
        step()
    torch.cuda.synchronize(device)
    g_step = capture(step, stream)
    # roofline graphs: the step's dominant launches alone (the fused layer
    # launches, or the attention launches of the two-launch path), and the
    # two-launch step itself for comparison
    if step.fused:
        g_attn = capture(lambda: [step.layer(i) for i in range(w.layers)], stream)
        g_pro = None
        step2 = DecodeStep(w, t, fused=False)
        with torch.cuda.stream(stream):
            step2()
        torch.cuda.synchronize(device)
        g_two = capture(step2, stream)
    else:
        g_attn = capture(lambda: [step.attention(i) for i in range(w.layers)], stream)
        g_pro = capture(lambda: [step.prologue(i) for i in range(w.layers)], stream)
        g_two = None

    clocks = ClockSampler(device.index)
    clocks.start()
    for _ in range(args.warmup):
        with torch.cuda.stream(stream):
            g_step.replay()
    torch.cuda.synchronize(device)
    barrier(world, device)
    torch.cuda.synchronize(device)
    ms_total = time_graph(g_step, args.steps, stream)
    torch.cuda.synchronize(device)
    barrier(world, device)
    clk = clocks.stop()
    ms_total = max_over_ranks(ms_total, world, device)
    ms_step = ms_total / args.steps

    # roofline of the dominant kernel: attention launches alone, same inputs
    reps = max(3, min(20, args.steps))
    ms_attn = time_graph(g_attn, reps, stream) / (reps * w.layers)
    ms_pro = time_graph(g_pro, reps, stream) / (reps * w.layers) if g_pro is not None else None
    ms_two = time_graph(g_two, reps, stream) / reps if g_two is not None else None
    # the fused launch also reads the new k/v and writes their slots
    attn_bytes = w.fused_bytes() if step.fused else w.attention_bytes()
    peaks = {}
    pk = REPO / "MEASURED_PEAKS.json"
    if pk.exists():
        peaks = json.loads(pk.read_text())
    peak = peaks.get("hbm_gbs")
    peak_src = "measured" if peak else "fallback"
    peak = peak or 6650.0
    achieved = attn_bytes / (ms_attn * 1e-3) / 1e9
    # DRAM traffic of the dominant launch, from a smaller capture of the same
    # kernel and workload, applied to this rank's algorithmic bytes per launch.
    traffic = _capture_traffic(full.name, step.fused, attn_bytes)

    e2e = None
    if not args.no_e2e:
        torch.cuda.synchronize(device)
        barrier(world, device)
        ms_e2e, h2d, d2h, _, e2e_mode = e2e_run(w, t, args.steps, args.warmup, device)
        barrier(world, device)
        ms_e2e = max_over_ranks(ms_e2e, world, device)
        e2e = {"value": full.batch / (ms_e2e * 1e-3), "unit": UNIT, "ms_per_step": ms_e2e,
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "path": "public ops with pinned host buffers; one H2D and one D2H copy per "
                       "layer group on copy streams (groups of 4 layers, single-layer first "
                       "and last groups), "
                       f"step launched as {'one CUDA graph' if e2e_mode == 'graph' else 'eager calls'}"}

    # the other even split, measured the same way (N > 1 only)
    alt = None
    if world > 1 and not args.no_alt:
        alt_mode = "contiguous" if args.sharding == "balanced" else "balanced"
        del g_step, g_attn, g_pro, g_two
        wa = full.shard(rank, world, alt_mode)
        ta = W.materialize(wa, device)
        step_a = DecodeStep(wa, ta)
        with torch.cuda.stream(stream):
            step_a()
        torch.cuda.synchronize(device)
        g_alt = capture(step_a, stream)
        for _ in range(args.warmup):
            with torch.cuda.stream(stream):
                g_alt.replay()
        torch.cuda.synchronize(device)
        barrier(world, device)
        ms_alt = max_over_ranks(time_graph(g_alt, args.steps, stream), world, device) / args.steps
        barrier(world, device)
        alt = {"sharding": alt_mode, "value": full.batch / (ms_alt * 1e-3), "ms_per_step": ms_alt,
               "max_rank_tokens": max_over_ranks(float(wa.lengths.sum()), world, device)}
        del g_alt, step_a, ta
        g_step = g_attn = g_pro = g_two = None

    # output checksum across ranks (outside every timed region)
    chk = torch.tensor([float(sum(o.float().abs().sum() for o in step.out))], device=device,
                       dtype=torch.float64)
    if world > 1:
        import torch.distributed as dist
        dist.all_reduce(chk)

    base = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        base = cpu_baseline(w, t)

    # the other configurations, after the headline workload's memory is freed
    step_fused, n_layers = step.fused, w.layers
    out_checksum = float(chk.item())
    secondary = None
    if not args.no_secondary and args.workload == "llama3_8b":
        del step, t, g_step, g_attn, g_pro, g_two
        torch.cuda.synchronize(device)
        torch.cuda.empty_cache()
        secondary = secondary_ours(args, device, world)

    if rank == 0:
        line = {
            "metric": METRIC, "value": full.batch / (ms_step * 1e-3), "unit": UNIT,
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f16" if full.dtype == torch.float16 else "f32",
            "data": "synthetic (seeded; no dataset in this path)",
            "config": decode_config(full, args, world),
            "step": ("per layer: decode_attention (RoPE + KV-slot write + attention in one "
                     "launch), one CUDA graph per step" if step_fused else
                     "per layer: rope_kv_write + paged_attention, one CUDA graph per step"),
            "algorithmic_gb_per_step": full.seq_step_bytes() / 1e9,
            "achieved_gbs_step": full.seq_step_bytes() / (ms_step * 1e-3) / 1e9,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic,
                         "kernel": attn_kernel_label(w.head_dim, step_fused, w.dtype),
                         "peak_source": f"{peak_src} hbm_gbs",
                         "algorithmic_bytes_per_launch": attn_bytes,
                         "ms_per_launch": ms_attn, "prologue_ms_per_launch": ms_pro,
                         "two_launch_ms_per_step": ms_two},
            "clocks": clk,
            "gpu_launches": args.steps * n_layers * (1 if step_fused else 2),
            "e2e": e2e,
            "cpu_baseline": base,
            "alt_sharding": alt,
            "checksum": out_checksum,
            "secondary": secondary,
        }
        print(json.dumps(line), flush=True)
    g_step = g_attn = g_pro = None
    if world > 1:
        import torch.distributed as dist
        dist.barrier(device_ids=[device.index])
        dist.destroy_process_group()


# The kernel a decode layer launches for an FP16 workload with GQA group <= 4
# (head_dim 128: 64-token tiles; head_dim 64: 128-token tiles, two 16-token
# blocks per warp), or the FP32 SIMT kernel.
def attn_kernel_label(head_dim: int, fused: bool, dtype: torch.dtype = torch.float16) -> str:
    if dtype == torch.float32:
        return (f"attn_tma_dyn_kernel<SimtMath<float,{head_dim},4,2,TMA>"
                f"{', fused prologue' if fused else ''}>: "
                f"{'RoPE + KV-slot write + attention, ' if fused else ''}FP32 SIMT inner loop "
                "(fp32 FMA throughout), TMA producer warp, stream-K with a dynamic tail, "
                "epilogue warp")
    m = "MmaMath<128,4,3,TMA>" if head_dim == 128 else f"MmaMath<{head_dim},4,3,TMA,2>"
    if fused:
        return (f"attn_tma_dyn_kernel<{m}, fused prologue>: RoPE + KV-slot write + attention, "
                "TMA producer warp, tensor-core stream-K, dynamic tail, epilogue warp")
    return (f"attn_tma_dyn_kernel<{m}>: TMA producer warp, tensor-core stream-K, dynamic "
            "tail, epilogue warp")


# --------------------------------------------------------------------------
# measurements shared by the headline line, its `secondary` object and the
# stand-alone --workload runs
# --------------------------------------------------------------------------
def _peaks() -> dict:
    pk = REPO / "MEASURED_PEAKS.json"
    return json.loads(pk.read_text()) if pk.exists() else {}


def _roofline(achieved: float, bound: str, kernel: str, **extra) -> dict:
    """Roofline entry against the measured peaks (burst figures: every kernel
    here is timed in launches of tens of microseconds to milliseconds)."""
    pk = _peaks()
    if bound == "hbm":
        peak, unit = pk.get("hbm_gbs"), "GB/s"
        src = "measured hbm_gbs" if peak else "fallback 6.65 TB/s"
        peak = peak or 6650.0
    else:
        peak, unit = pk.get("bf16_tflops"), "TFLOP/s"
        src = "measured bf16_tflops (burst)" if peak else "fallback 1.59 PFLOP/s"
        peak = peak or 1590.0
    return {"bound": bound, "achieved": achieved, "peak": peak, "unit": unit,
            "frac": achieved / peak, "traffic": None, "kernel": kernel, "peak_source": src,
            **extra}


def timed_replays(run, stream, device, units: int, min_s: float = 0.3, max_reps: int = 200):
    """Median ms per unit over back-to-back timed replays of `run` (each
    replay does `units` units of work, bracketed by CUDA events on `stream`),
    repeated until `min_s` seconds have passed so that the clock sampler sees
    the timed region; clocks are sampled throughout."""
    clocks = ClockSampler(device.index)
    clocks.start()
    times, t_end = [], time.perf_counter() + min_s
    while (time.perf_counter() < t_end and len(times) < max_reps) or len(times) < 3:
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            s.record(stream)
            run()
            e.record(stream)
        e.synchronize()
        times.append(s.elapsed_time(e) / units)
    return statistics.median(times), clocks.stop(), len(times)


def _capture_traffic(workload: str, fused: bool, algorithmic_bytes: float):
    """DRAM bytes (read + write) of one launch: the ncu traffic /
    algorithmic-bytes ratio of a committed capture of the same kernel and
    workload (profiles/traffic_*.json; a full launch is often too large for a
    multi-pass capture, and traffic grows with the K/V bytes read), applied
    to these algorithmic bytes. None without such a capture."""
    for f in sorted((REPO / "profiles").glob("traffic_*.json")):
        tj = json.loads(f.read_text())
        if (tj.get("workload") == workload and tj.get("fused", True) == fused
                and tj.get("ratio_to_algorithmic")):
            return int(round(tj["ratio_to_algorithmic"] * algorithmic_bytes))
    return None


def measure_decode(w, device, steps: int, warmup: int) -> dict:
    """Decode steps of workload `w` (every layer: RoPE + KV-slot write +
    attention) through the public ops, one CUDA graph per step, K steps per
    timed replay; the step's attention launches replayed alone give the
    roofline figure. Inputs are larger than L2 (all layers' pools)."""
    t = W.materialize(w, device)
    step = DecodeStep(w, t)
    stream = torch.cuda.Stream(device)
    with torch.cuda.stream(stream):
        step()
    torch.cuda.synchronize(device)
    g_step = capture(step, stream)
    g_dom = g_step if step.fused else capture(
        lambda: [step.attention(i) for i in range(w.layers)], stream)
    for _ in range(warmup):
        with torch.cuda.stream(stream):
            g_step.replay()
    torch.cuda.synchronize(device)

    def k_steps():
        for _ in range(steps):
            g_step.replay()
    ms, clk, reps = timed_replays(k_steps, stream, device, steps)
    ms_launch, _, _ = timed_replays(g_dom.replay, stream, device, w.layers, min_s=0.05)
    nbytes = w.fused_bytes() if step.fused else w.attention_bytes()
    kernel = attn_kernel_label(w.head_dim, step.fused, w.dtype)
    pools_gb = 2 * w.layers * w.num_blocks * w.block_size * w.kv_heads * w.head_dim \
        * w.elem_bytes / 1e9
    res = {"metric": METRIC, "value": w.batch / (ms * 1e-3), "unit": UNIT, "ms_per_step": ms,
           "ms_per_launch": ms_launch, "dtype": "f16" if w.dtype == torch.float16 else "f32",
           "config": {"workload": f"{w.name}: batch {w.batch}, {w.heads}/{w.kv_heads} heads, "
                                  f"head_dim {w.head_dim}, {w.layers} layers, block "
                                  f"{w.block_size}", "batch": w.batch, "layers": w.layers,
                      "max_length": w.max_length,
                      "mean_length": float(w.lengths.float().mean()),
                      "l2": "inputs larger than L2 (KV pools %.1f GB)" % pools_gb},
           "step": ("per layer: decode_attention (one launch)" if step.fused else
                    "per layer: rope_kv_write + paged_attention (two launches)"),
           "timing": f"median of {reps} CUDA-event-timed replays of {steps} graph steps",
           "roofline": _roofline(nbytes / (ms_launch * 1e-3) / 1e9, "hbm", kernel,
                                 algorithmic_bytes_per_launch=nbytes, ms_per_launch=ms_launch),
           "clocks": clk, "gpu_launches": steps * w.layers * (1 if step.fused else 2)}
    res["roofline"]["traffic"] = _capture_traffic(w.name, step.fused, nbytes)
    del g_step, g_dom, step, t
    torch.cuda.empty_cache()
    return res


def measure_decode_reference(w, device, steps: int, mod) -> dict:
    """The reference's decode attention on this GPU for workload `w`, as its
    PagedLlama.decode runs it per layer: RoPE in torch ops
    (worker/llama.py:108-117), the two slot writes (:171-172) and its own CUDA
    kernel (cuda/paged_attention.cu:10-74, built from the reference's sources
    into oracle/_ref), launched eagerly as the reference launches them. The
    kernel alone is timed too (one launch per layer on the same pools)."""
    from oracle import kv_cache, rope as orope
    t = W.materialize(w, device)
    pos, phys, off = t.positions, t.physical, t.offsets

    def attention(layer, q):
        return mod.paged_attention(q.contiguous(), t.k_pools[layer], t.v_pools[layer],
                                   t.tables, t.lengths, w.max_length)

    def step():
        for layer in range(w.layers):
            qr, kr = orope.rope(t.q[layer].unsqueeze(1), t.k[layer].unsqueeze(1), pos,
                                t.inv_freq)
            kv_cache.write_decode(t.k_pools[layer], phys, off, kr[:, 0])
            kv_cache.write_decode(t.v_pools[layer], phys, off, t.v[layer])
            attention(layer, qr[:, 0])

    def kernels():
        for layer in range(w.layers):
            attention(layer, t.q[layer])
    stream = torch.cuda.current_stream(device)
    step()
    torch.cuda.synchronize(device)
    ms, clk, reps = timed_replays(step, stream, device, 1, min_s=0.3, max_reps=max(steps, 3))
    ms_launch, _, _ = timed_replays(kernels, stream, device, w.layers, min_s=0.1,
                                    max_reps=max(steps, 3))
    nbytes = w.attention_bytes()
    res = {"metric": METRIC, "value": w.batch / (ms * 1e-3), "unit": UNIT, "ms_per_step": ms,
           "ms_per_launch": ms_launch, "config": {"workload": w.name, "batch": w.batch,
                                                  "layers": w.layers},
           "step": "per layer: PagedLlama.rope (torch ops), two index_put slot writes, the "
                   "reference's CUDA kernel; eager launches",
           "timing": f"median of {reps} CUDA-event-timed steps",
           "roofline": _roofline(nbytes / (ms_launch * 1e-3) / 1e9, "hbm",
                                 "reference attention_kernel (cuda/paged_attention.cu), one CTA "
                                 "per (sequence, head)", algorithmic_bytes_per_launch=nbytes),
           "clocks": clk}
    del t
    torch.cuda.empty_cache()
    return res


def _reference_kernel_module():
    """The reference's own CUDA kernel, prebuilt into oracle/_ref (None when
    it was not built)."""
    from oracle import build_ref
    return build_ref.load_ref_module()


# --------------------------------------------------------------------------
# the reference arm: the reference's own CPU path, timed on the host cores
# --------------------------------------------------------------------------
def run_reference(args):
    """The reference's own CPU implementation of the path (oracle port of
    worker/llama.py:58-71, :108-117, :171-172; the reference compiles no CPU
    code) on the host cores, same workload, metric and config. One step is a
    bounded sample: 4 sequences through one layer, the same for every layer
    (all layers have identical shapes and lengths), so seq-steps/s =
    4 / (step time x layers). At N = 1 the line also carries the reference's
    own GPU code timed on this box (its CUDA kernel and torch paths) for the
    headline and the other configurations."""
    world, rank, local = dist_env()
    if rank != 0:
        return
    from oracle import kv_cache, paged_attention as opa, rope as orope
    torch.set_num_threads(os.cpu_count() or 1)
    full = make_workload(args)
    n = min(4, full.batch)
    tabs, blocks, used = W.make_decode_tables(full.lengths[:n], full.block_size, full.seed, 1.25, None)
    # pad the sample's tables to the batch's width, as TensorPagedKV.metadata does
    wide = torch.zeros(n, full.table_width, dtype=torch.int32)
    wide[:, :tabs.shape[1]] = tabs
    sub = W.DecodeWorkload(full.name, n, full.heads, full.kv_heads, full.head_dim, 1,
                           full.block_size, full.dtype, full.theta, full.seed, full.lengths[:n],
                           wide, blocks, used, stale_scale=full.stale_scale)
    t = W.materialize(sub, "cpu")
    pos = sub.positions()
    phys, off = sub.slots()
    times = []
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        qr, kr = orope.rope(t.q[0].unsqueeze(1), t.k[0].unsqueeze(1), pos, t.inv_freq)
        kv_cache.write_decode(t.k_pools[0], phys, off, kr[:, 0])
        kv_cache.write_decode(t.v_pools[0], phys, off, t.v[0])
        opa.paged_attention(qr[:, 0], t.k_pools[0], t.v_pools[0], sub.tables, sub.lengths,
                            full.max_length)
        if i >= args.warmup:
            times.append(time.perf_counter() - t0)
    sec = sum(times) / len(times)  # one sample step: n sequences through one layer
    value = n / (sec * full.layers)
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic (seeded; no dataset in this path)", "impl": "reference",
            "config": decode_config(full, args, world),
            "step": f"a bounded sample: {n} of {full.batch} sequences through one layer "
                    "(RoPE, slot writes, gather + repeat + masked SDPA), padded to the "
                    f"batch's max_length {full.max_length}",
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": torch.get_num_threads(),
                             "kind": "port",
                             "sample": f"{n} of {full.batch} sequences x 1 layer per step, "
                                       f"scaled by {full.layers} layers; padded to max_length "
                                       f"{full.max_length}; os.cpu_count()={os.cpu_count()}"},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    if world == 1 and torch.cuda.is_available() and not args.no_secondary:
        device = torch.device("cuda", local)
        torch.cuda.set_device(device)
        mod = _reference_kernel_module()
        if mod is None:
            line["reference_cuda"] = {"unavailable": "the reference kernel was not built "
                                                     "into oracle/_ref"}
        else:
            line["reference_cuda"] = measure_decode_reference(full, device, 3, mod)
        line["secondary"] = secondary_reference(args, device, mod)
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------
# decode tick of the SmolLM2-135M architecture (the model runner)
# --------------------------------------------------------------------------
TICK_METRIC = "decode tokens/s (SmolLM2-135M arch, 128 sequences, len U[16,4096])"
TICK_UNIT = "tokens/s"
TICK_SEED_MODEL, TICK_SEED_STATE = 2024, 5


def _init_dist(device, world):
    if world > 1:
        import datetime
        import torch.distributed as dist
        if not dist.is_initialized():
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=device)


def _tick_inputs(B, steps, warmup, device):
    if steps + max(warmup, 3) > 200:
        raise SystemExit("smollm_tick: steps + warmup must stay within the 256 reserved tokens")
    cfg = W.smollm2_135m_config()
    model = W.seeded_llama(cfg, TICK_SEED_MODEL, torch.float16, device)
    blocks = W.tick_blocks(B, TICK_SEED_STATE)
    g = torch.Generator().manual_seed(99)
    toks = torch.randint(0, cfg.vocab_size, (warmup + 2 * steps + 4, B), generator=g)
    return cfg, model, blocks, toks


def _tick_bytes(cfg, lengths, model) -> float:
    """Algorithmic HBM bytes of one tick: every weight once, every cached K/V
    row of every layer once (2 * len * kv_heads * head_dim * 2 bytes)."""
    weights = sum(p.numel() for p in model.parameters()) * 2
    kv = 2 * float(lengths.sum()) * cfg.num_key_value_heads * cfg.head_dim * 2
    return weights + kv * cfg.num_hidden_layers


def _tick_e2e(runner, ids, toks, start, steps, device):
    """``steps`` ticks through the public API: token ids in (H2D), greedy next
    token out (D2H), CUDA events on the current stream; returns ms per tick."""
    nxt = toks[start].tolist()
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        logits = runner.decode(ids, nxt)
        nxt = logits.argmax(-1).tolist()
    e1.record()
    e1.synchronize()
    return e0.elapsed_time(e1) / steps


def measure_tick(device, world, steps: int, warmup: int, B: int = 128) -> dict:
    """One replica per GPU: the decode tick of the SmolLM2-135M architecture
    through llama_runner.PagedLlama with graph-captured ticks, device time of
    K replays (max over ranks), then K ticks end to end through
    PagedLlama.decode with greedy sampling to the host."""
    cfg, model, blocks, toks = _tick_inputs(B, steps, warmup, device)
    runner = PKG.PagedLlama(model, None, blocks=blocks, block_size=16, max_batch=B, graphs=True)
    ids, lengths = W.decode_tick_state(runner.cache, B, TICK_SEED_STATE)
    for i in range(max(warmup, 3)):  # eager tick, capture, replays
        runner.decode(ids, toks[i].tolist())
    torch.cuda.synchronize(device)
    tick = runner._b200_graphs[B]
    with torch.inference_mode():  # the graph's buffers were made in inference mode
        tick.tokens.copy_(toks[0].view(B, 1))
    clocks = ClockSampler(device.index)
    clocks.start()
    barrier(world, device)
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        tick.graph.replay()
    e1.record()
    e1.synchronize()
    clk = clocks.stop()
    ms_tick = max_over_ranks(e0.elapsed_time(e1) / steps, world, device)
    # the replays advanced the device lengths past the host's: re-upload them
    runner.cache._rows = [None] * runner.cache.max_batch
    barrier(world, device)
    ms_e2e = max_over_ranks(_tick_e2e(runner, ids, toks, max(warmup, 3), steps, device),
                            world, device)
    ms_attn = _time_attention_share(runner, B, device)
    nbytes = _tick_bytes(cfg, lengths + max(warmup, 3), model)
    res = {
        "metric": TICK_METRIC, "value": world * B / (ms_tick * 1e-3), "unit": TICK_UNIT,
        "ms_per_step": ms_tick, "scaling": "weak", "dtype": "f16",
        "config": {"workload": "smollm2-135m decode tick: 30 layers, 9/3 heads, head_dim 64, "
                               f"hidden 576, vocab 49152, batch {B} per GPU, lengths "
                               "U[16,4096], pages reused in shuffled order, block 16",
                   "batch_per_gpu": B, "mean_length": float(lengths.float().mean()),
                   "parallelism": f"replica x{world}",
                   "l2": "inputs larger than L2 (KV %.1f GB)" % (
                       2 * runner.cache.keys.numel() * 2 / 1e9)},
        "step": "one CUDA graph per tick: embedding, 30 x (norm, fused q/k/v GEMM, "
                "decode_attention, o GEMM, MLP), norm, LM head",
        "roofline": _roofline(nbytes / (ms_tick * 1e-3) / 1e9, "hbm",
                              "whole tick (weights once + every cached K/V row once)",
                              algorithmic_bytes_per_step=nbytes,
                              attention_ms_per_step=ms_attn),
        "clocks": clk,
        "gpu_launches": steps * cfg.num_hidden_layers,
        "e2e": {"value": world * B / (ms_e2e * 1e-3), "unit": TICK_UNIT,
                "ms_per_step": ms_e2e, "h2d_bytes_per_step": B * 8,
                "d2h_bytes_per_step": B * 8,
                "path": "PagedLlama.decode(ids, tokens) per tick, greedy next token to "
                        "the host"},
    }
    del runner, tick, model
    torch.cuda.empty_cache()
    return res


def measure_tick_reference(device, steps: int, warmup: int, mod, B: int = 128) -> dict:
    """The reference decode tick (worker/llama.py:151-177, restated and pinned
    in oracle/llama_model.py) with its own CUDA attention kernel (or its torch
    path when that kernel was not built), same model, state and loop."""
    from oracle import llama_model as LM
    cfg, model, blocks, toks = _tick_inputs(B, steps, warmup, device)
    if mod is not None:
        def attention(q, k, v, tables, lengths, max_length):
            return mod.paged_attention(q.contiguous(), k, v, tables.contiguous(),
                                       lengths.contiguous(), max_length)
        which = "reference CUDA kernel (cuda/paged_attention.cu, built into oracle/_ref)"
    else:
        attention, which = None, "reference torch path (torch_paged_attention)"
    runner = LM.PagedLlamaOracle(model, blocks=blocks, block_size=16, attention=attention)
    ids, lengths = W.decode_tick_state(runner.cache, B, TICK_SEED_STATE)
    for i in range(max(warmup, 3)):
        runner.decode(ids, toks[i].tolist())
    clocks = ClockSampler(device.index)
    clocks.start()
    ms = _tick_e2e(runner, ids, toks, max(warmup, 3), steps, device)
    clk = clocks.stop()
    res = {"metric": TICK_METRIC, "value": B / (ms * 1e-3), "unit": TICK_UNIT,
           "ms_per_step": ms, "scaling": "weak", "dtype": "f16",
           "config": {"workload": "smollm2-135m decode tick", "batch_per_gpu": B,
                      "attention": which, "parallelism": "replica x1"},
           "clocks": clk,
           "e2e": {"value": B / (ms * 1e-3), "unit": TICK_UNIT, "ms_per_step": ms,
                   "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    del runner, model
    torch.cuda.empty_cache()
    return res


def run_tick(args):
    world, rank, local = dist_env()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    _init_dist(device, world)
    B = args.batch or 128
    if args.impl == "reference":
        res = measure_tick_reference(device, args.steps, args.warmup, _reference_kernel_module(), B)
        res["impl"] = "reference"
    else:
        res = measure_tick(device, world, args.steps, args.warmup, B)
    if rank == 0:
        line = {"n_gpus": world, "steps": args.steps, "warmup": max(args.warmup, 3),
                "higher_is_better": True, "vs_baseline": None,
                "data": "synthetic (seeded random-init weights and KV; no checkpoint)", **res}
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.barrier(device_ids=[device.index])
        dist.destroy_process_group()


def _time_attention_share(runner, B, device, reps=10):
    """Attention launches of one tick alone (same pools, tables and lengths)."""
    cache = runner.cache
    q = torch.randn(B, runner.heads, runner.head_dim, device=device, dtype=runner.dtype)
    tables, lengths = cache.dev_tables[:B], cache.dev_lengths[:B]
    out = torch.empty_like(q)
    layers = cache.keys.size(0)

    def run():
        for i in range(layers):
            PKG.paged_attention(q, cache.keys[i], cache.values[i], tables, lengths,
                                cache.max_tokens, out=out)
    stream = torch.cuda.Stream(device)
    with torch.cuda.stream(stream):
        run()
    torch.cuda.synchronize(device)
    g = capture(run, stream)
    return time_graph(g, reps, stream) / reps


# --------------------------------------------------------------------------
# prefill attention (16 prompts, SmolLM2 heads)
# --------------------------------------------------------------------------
PREFILL_METRIC = "prefill attention prompt tokens/s per layer (16 prompts, len U[64,1024])"
# Independent copies of a prefill step's inputs; consecutive steps use
# different copies, so the timed steps read more than L2 holds.
L2_COPIES = 4


def _prefill_case(device, B=16, H=9, KVH=3, D=64, bs=16, seed=4):
    g = torch.Generator().manual_seed(seed)
    lengths = torch.randint(64, 1025, (B,), generator=g)
    Wd = int(lengths.max())
    pages = ((lengths + bs - 1) // bs).tolist()
    N = int(1.25 * sum(pages))
    perm = torch.randperm(N, generator=g)
    tables = torch.zeros(B, max(pages), dtype=torch.int32)
    off = 0
    for b, n in enumerate(pages):
        tables[b, :n] = perm[off:off + n].to(torch.int32)
        off += n
    q = torch.randn(B, Wd, H, D, generator=g).half().to(device)
    k = torch.randn(B, Wd, KVH, D, generator=g).half().to(device)
    v = torch.randn(B, Wd, KVH, D, generator=g).half().to(device)
    valid = (torch.arange(Wd)[None, :] < lengths[:, None]).to(device)
    tok = torch.arange(Wd)[None, :].expand(B, -1)
    phys = tables.long().gather(1, (tok // bs).clamp(max=tables.shape[1] - 1)).to(device)
    offs = (tok % bs).to(device)
    k_pool = torch.randn(N, bs, KVH, D, generator=g).half().to(device)
    v_pool = torch.randn(N, bs, KVH, D, generator=g).half().to(device)
    k_pool[phys[valid], offs[valid]] = k[valid]
    v_pool[phys[valid], offs[valid]] = v[valid]
    flops = float(sum(n * (n + 1) // 2 for n in lengths.tolist())) * H * D * 4
    return dict(q=q, k=k, v=v, k_pool=k_pool, v_pool=v_pool, tables=tables.to(device),
                lengths=lengths.to(torch.int32).to(device), tokens=int(lengths.sum()),
                flops=flops, H=H, KVH=KVH, D=D)


def _graph_of_steps(step_fns, steps, stream, device, warmup):
    """One CUDA graph of `steps` steps, step i running step_fns[i % len]."""
    with torch.cuda.stream(stream):
        for _ in range(max(warmup, 1)):
            for fn in step_fns:
                fn()
    torch.cuda.synchronize(device)

    def run():
        for i in range(steps):
            step_fns[i % len(step_fns)]()
    g = capture(run, stream)
    time_graph(g, 1, stream)  # graph upload
    return g


def measure_prefill(device, steps: int, warmup: int, impl: str = "ours",
                    kernel: str = "auto") -> dict:
    cases = [_prefill_case(device) for _ in range(L2_COPIES)]
    c0 = cases[0]
    if impl == "reference":
        import torch.nn.functional as F
        groups = c0["H"] // c0["KVH"]

        def make(c):
            def step():  # worker/llama.py:141-144
                ctx = F.scaled_dot_product_attention(
                    c["q"].transpose(1, 2),
                    c["k"].repeat_interleave(groups, dim=2).transpose(1, 2),
                    c["v"].repeat_interleave(groups, dim=2).transpose(1, 2), is_causal=True)
                return ctx.transpose(1, 2).reshape(c["q"].shape[0], c["q"].shape[1], -1)
            return step
        which = "reference prefill attention: repeat_interleave + causal SDPA on the padded batch"
    else:
        impl_id = {"auto": PKG.PREFILL_AUTO, "tcgen05": PKG.PREFILL_TCGEN05,
                   "mma": PKG.PREFILL_MMA}[kernel]

        def make(c):
            out = torch.empty_like(c["q"])

            def step():
                return PKG.prefill_attention(c["q"], c["k_pool"], c["v_pool"], c["tables"],
                                             c["lengths"], out=out, impl=impl_id)
            return step
        which = ("prefill_attention_kernel<64> (mma.sync; K/V from the paged pools)"
                 if kernel == "mma" else
                 "prefill_tc_kernel<64> (tcgen05.mma + TMEM, TMA from the paged pools)")
    stream = torch.cuda.Stream(device)
    g = _graph_of_steps([make(c) for c in cases], steps, stream, device, warmup)
    ms, clk, reps = timed_replays(g.replay, stream, device, steps)
    tflops = c0["flops"] / (ms * 1e-3) / 1e12
    res = {"metric": PREFILL_METRIC, "value": c0["tokens"] / (ms * 1e-3), "unit": "tokens/s",
           "ms_per_step": ms, "scaling": "replicas only", "dtype": "f16",
           "config": {"workload": "prefill attention: 16 prompts, len U[64,1024], heads 9/3, "
                                  "head_dim 64, block 16, one layer per step",
                      "prompt_tokens": c0["tokens"],
                      "l2": f"{L2_COPIES} input copies used in turn (inputs larger than L2)"},
           "timing": f"median of {reps} CUDA-event-timed replays of a {steps}-step graph",
           "roofline": _roofline(tflops, "tensor", which, algorithmic_flops_per_step=c0["flops"],
                                 note="causal FLOPs only (QK and PV over keys <= query)"),
           "clocks": clk, "gpu_launches": steps if impl != "reference" else None}
    del g, cases
    torch.cuda.empty_cache()
    return res


def run_prefill(args):
    world, rank, local = dist_env()
    if rank != 0:
        return
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    res = measure_prefill(device, args.steps, args.warmup, args.impl, args.prefill_kernel)
    line = {"n_gpus": 1, "steps": args.steps, "warmup": max(args.warmup, 3),
            "higher_is_better": True, "vs_baseline": None, "data": "synthetic (seeded)", **res}
    if args.impl == "reference":
        line["impl"] = "reference"
    print(json.dumps(line), flush=True)


PREFILL_WRITE_METRIC = ("prefill RoPE + paged KV write prompt tokens/s per layer "
                        "(16 prompts, len U[64,1024])")


def measure_prefill_write(device, steps: int, warmup: int, impl: str = "ours") -> dict:
    """Prefill RoPE + paged KV-slot write of one layer (worker/llama.py:128-140),
    16 SmolLM2-shaped prompts padded to the longest, into a 4096-block pool.
    Ours: rope_kv_write with the valid mask (one varlen launch). Reference:
    the reference's torch steps on the same GPU — RoPE of the padded q/k with
    every op in FP16 (worker/llama.py:108-117) and pool[slots] = k[valid],
    v[valid] (:138-140); the valid rows' flat indices are computed once,
    outside the timed steps."""
    pw = W.prefill_smollm()
    copies = [W.materialize_prefill(pw, device) for _ in range(L2_COPIES)]
    d0 = copies[0]
    B, Wd, H, D = d0["q"].shape
    KVH = d0["k"].shape[2]
    e = d0["q"].element_size()
    ntok = int(pw.lengths.sum())
    nbytes = ((2 * B * Wd * H * D + 3 * B * Wd * KVH * D) * e  # read q, k, v; write q', k'
              + 2 * ntok * KVH * D * e + B * Wd)                # k, v slot writes; mask
    if impl == "reference":
        def rot(x):
            a, b = x.chunk(2, dim=-1)
            return torch.cat((-b, a), dim=-1)

        def make(d):
            vidx = d["valid"].reshape(-1).nonzero()[:, 0]
            q_o, k_o = torch.empty_like(d["q"]), torch.empty_like(d["k"])

            def step():
                f = d["positions"].float()[..., None] * d["inv_freq"]
                ang = torch.cat((f, f), dim=-1)
                cos = ang.cos().to(d["q"].dtype).unsqueeze(2)
                sin = ang.sin().to(d["q"].dtype).unsqueeze(2)
                torch.add(d["q"] * cos, rot(d["q"]) * sin, out=q_o)
                torch.add(d["k"] * cos, rot(d["k"]) * sin, out=k_o)
                d["k_pool"][d["physical"], d["offsets"]] = k_o.view(-1, KVH, D)[vidx]
                d["v_pool"][d["physical"], d["offsets"]] = d["v"].view(-1, KVH, D)[vidx]
            return step
        which = "reference prefill RoPE (torch ops in FP16) + index_put of the valid rows"
    else:
        def make(d):
            q_o, k_o = torch.empty_like(d["q"]), torch.empty_like(d["k"])

            def step():
                PKG.rope_kv_write(d["q"], d["k"], d["v"], d["k_pool"], d["v_pool"],
                                  d["physical"], d["offsets"], d["positions"], d["inv_freq"],
                                  valid=d["valid"], q_out=q_o, k_out=k_o)
            return step
        which = ("valid_scan_kernel + rope_prefill_vec_kernel (rows staged in shared memory, "
                 "varlen scatter into the pages)")
    stream = torch.cuda.Stream(device)
    g = _graph_of_steps([make(d) for d in copies], steps, stream, device, warmup)
    ms, clk, reps = timed_replays(g.replay, stream, device, steps)
    gbs = nbytes / (ms * 1e-3) / 1e9
    res = {"metric": PREFILL_WRITE_METRIC, "value": ntok / (ms * 1e-3), "unit": "tokens/s",
           "ms_per_step": ms, "scaling": "replicas only", "dtype": "f16",
           "config": {"workload": "prefill RoPE + KV write: 16 prompts, len U[64,1024], heads "
                                  "9/3, head_dim 64, block 16, 4096-block pool, one layer per "
                                  "step", "prompt_tokens": ntok,
                      "l2": f"{L2_COPIES} input copies used in turn (inputs larger than L2)"},
           "timing": f"median of {reps} CUDA-event-timed replays of a {steps}-step graph",
           "roofline": _roofline(gbs, "hbm", which, algorithmic_bytes_per_step=nbytes,
                                 note="padded q, k, v read and q', k' written; valid rows' "
                                      "k/v slots"),
           "clocks": clk, "gpu_launches": 2 * steps if impl != "reference" else None}
    del g, copies
    torch.cuda.empty_cache()
    return res


def run_prefill_write(args):
    world, rank, local = dist_env()
    if rank != 0:
        return
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    res = measure_prefill_write(device, args.steps, args.warmup, args.impl)
    line = {"n_gpus": 1, "steps": args.steps, "warmup": max(args.warmup, 3),
            "higher_is_better": True, "vs_baseline": None, "data": "synthetic (seeded)", **res}
    if args.impl == "reference":
        line["impl"] = "reference"
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------
# the other configurations, measured in the same run as the headline
# --------------------------------------------------------------------------
def secondary_ours(args, device, world) -> dict:
    """Every other configuration in the same run, each with its own CUDA-event
    time, roofline figure and clock record. At N = 1: the SmolLM2 decode in
    FP16 (30 pools) and FP32, the prefill RoPE + KV write, the prefill
    attention and the decode tick. At N > 1 the decode tick alone, one replica
    per GPU (weak scaling, max over ranks)."""
    out = {}
    steps, warmup = args.steps, args.warmup
    if world == 1:
        out["smollm_fp16"] = measure_decode(W.smollm_fp16(), device, steps, warmup)
        out["smollm_fp32"] = measure_decode(W.smollm_fp32(), device, steps, warmup)
        out["prefill_write"] = measure_prefill_write(device, steps, warmup)
        out["prefill_attention"] = measure_prefill(device, steps, warmup)
    out["decode_tick"] = measure_tick(device, world, min(steps, 100), warmup)
    return out


def secondary_reference(args, device, mod) -> dict:
    """The reference's own code for the same configurations, on the same GPU:
    its decode layer (torch RoPE, slot writes, its CUDA kernel) for the
    SmolLM2 shapes, its prefill RoPE + slot writes and prefill attention in
    torch, and its PagedLlama.decode tick with its CUDA kernel."""
    out = {}
    steps, warmup = args.steps, args.warmup
    if mod is not None:
        out["smollm_fp16"] = measure_decode_reference(W.smollm_fp16(), device, 3, mod)
        out["smollm_fp32"] = measure_decode_reference(W.smollm_fp32(), device, 3, mod)
    out["prefill_write"] = measure_prefill_write(device, steps, warmup, "reference")
    out["prefill_attention"] = measure_prefill(device, steps, warmup, "reference")
    out["decode_tick"] = measure_tick_reference(device, min(steps, 10), warmup, mod)
    return out


def main():
    args = parse()
    if args.workload == "prefill":
        run_prefill(args)
    elif args.workload == "prefill_write":
        run_prefill_write(args)
    elif args.workload == "smollm_tick":
        run_tick(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
