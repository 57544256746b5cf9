#!/usr/bin/env python
"""MXFP8 grouped-GEMM benchmark: TFLOPS geomean over the 36 Llama4 shapes x
{forward, dgrad, wgrad} on B200, printed as one JSON line.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl mxgg|reference]

* Shapes and offsets follow the reference bench (bench.py:113-122, 243-257):
  E in {1,2,4,8}, M = 16640 tokens, N, K in {2048, 5120, 8192}; offsets from
  ``generate_jagged_offs(E, M, 32)`` after ``random.seed(123)`` in the same
  shape order.  Inputs are seeded synthetic bf16 ~N(0,1), quantised on the
  GPU outside the timed region (the reference times the GEMM only).
* One step = one pass over all 108 (shape, pass) GEMMs.  Each call (scale
  pack + GEMM, captured once as a CUDA graph so host overhead stays out of
  the device timing) is preceded by an L2 flush (a 512 MiB memset, outside
  the events) and bracketed by CUDA events on the launching stream.
* TFLOPS = 2*M*N*K / t per (shape, pass) (bench.py:200); ``value`` is the
  geomean over the 108 points, times N for N > 1.
* N > 1 (one process per GPU): the same sweep, expert parallel.  Every rank
  holds M tokens (the single-GPU group sizes, rotated by rank so every rank
  computes M rows: weak scaling).  fwd and dgrad stream their rows to the
  hosting ranks over NVLink and send the output tiles back from the GEMM's
  epilogue (``mxgg.ep.FusedExpertParallel``; ``--ep-impl nccl`` for the NCCL
  all-to-all baseline).  wgrad runs on the hosting rank; replicated experts
  (E < N) sum their gradients in place over peer memory
  (``mxgg.ep.ReplicaSum``; an NCCL all-reduce with ``--ep-impl nccl``).
  Times are the max over ranks;
  ``expert_parallel`` splits them into phases.
* ``moe_layer``: BASELINE config 5, weak-scaled (8 experts and 16384 tokens
  per GPU; 64 and 131072 at 8 GPUs): a top-2 MoE layer forward, up
  5120 -> 8192 and down 8192 -> 5120, with MXFP8 weights and with MXFP4
  weights.  ``mxfp4_weights`` (1 GPU): the 36 forward shapes with e2m1
  weights.
* ``e2e``: the same geomean measured through the public entry points with
  host (pinned) inputs: H2D of the fp8 operands, scales and offsets, the GEMM,
  and D2H of the output, all inside the events.  On one GPU each call goes
  through ``mxgg.host.HostPipeline``: eight pieces on three streams, so the
  copies overlap the GEMM pieces (bit-identical results).
* ``--impl reference``: the reference's CPU path (dequantise + per-group fp32
  matmul, the oracle restatement -- the reference's Triton kernels are
  ROCm-only) timed on this host's cores over a bounded sample.
* ``--torch-arm`` (1 GPU): adds ``torch_scaled_grouped_mm``, torch's own
  MXFP8 grouped GEMM timed beside this library's on the same forward points.
"""

import argparse
import json
import math
import os
import random
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "grouped-gemms_b200"))
sys.path.insert(0, ROOT)

METRIC = "MXFP8 grouped-GEMM TFLOPS geomean, 36 shapes fwd/dgrad/wgrad, % of B200 peak"
NOMINAL_MXFP8_TFLOPS = 4500.0
M_TOKENS = 16640


def llama4_shapes():
    return [(e, M_TOKENS, n, k) for e in (1, 2, 4, 8) for n in (2048, 5120, 8192) for k in (2048, 5120, 8192)]


def geomean(xs):
    xs = [x for x in xs if x > 0 and math.isfinite(x)]
    return math.exp(sum(math.log(x) for x in xs) / len(xs)) if xs else float("nan")


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """SM clock and clock-event reasons while the timed region runs: NVML
    polled every 20 ms (the library nvidia-smi reads; read-only queries), or
    `nvidia-smi -lms 200` where the NVML bindings are missing.  A short
    multi-GPU timed region can end before nvidia-smi has printed a sample,
    which is why NVML comes first."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASON_NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, device_index):
        self.idx = device_index
        self.proc = None
        self.lines = []
        self.samples = []          # NVML: (sm MHz, max sm MHz, reason names)
        self.source = None
        self._stop = threading.Event()
        self.t = None

    def _nvml_start(self):
        import pynvml as nv
        nv.nvmlInit()
        h = nv.nvmlDeviceGetHandleByUUID(self.idx) if str(self.idx).startswith("GPU-") \
            else nv.nvmlDeviceGetHandleByIndex(int(self.idx))
        bits = {"hw_slowdown": nv.nvmlClocksEventReasonHwSlowdown,
                "hw_thermal_slowdown": nv.nvmlClocksEventReasonHwThermalSlowdown,
                "sw_thermal_slowdown": nv.nvmlClocksEventReasonSwThermalSlowdown,
                "sw_power_cap": nv.nvmlClocksEventReasonSwPowerCap}
        mx = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
        nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)            # fails here, not in the thread

        def poll():
            while not self._stop.is_set():
                try:
                    sm = float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
                    r = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                    self.samples.append((sm, mx, tuple(n for n, b in bits.items() if r & b)))
                except Exception:
                    pass
                self._stop.wait(0.02)
            try:
                nv.nvmlShutdown()
            except Exception:
                pass

        self.t = threading.Thread(target=poll, daemon=True)
        self.t.start()
        self.source = "nvml"

    def __enter__(self):
        try:
            self._nvml_start()
            return self
        except Exception:
            self.source = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.idx)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            self.source = "nvidia-smi"
            # nvidia-smi can take a second or more to start on a many-GPU box,
            # longer than a short timed region: wait for its first sample (taken
            # before the load starts, so it is dropped)
            t0 = time.time()
            while not self.lines and self.proc.poll() is None and time.time() - t0 < 15:
                time.sleep(0.05)
            self.lines.clear()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        self._stop.set()
        if self.source == "nvml" and self.t is not None:
            self.t.join(timeout=5)
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        for (s_, m_, rs) in self.samples:
            sm.append(s_)
            mx = m_
            reasons.update(rs)
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(self.REASON_NAMES, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0, "source": self.source}
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm),
                "source": self.source}


# ------------------------------------------------------------------ inputs
def build_problems(device, shapes, passes, seed=123, multiple_of=32, scale_layout="row_major"):
    """Quantised operands for every (shape, pass); offsets as the reference draws them
    (group sizes multiples of `multiple_of`; wgrad needs 32).  scale_layout
    "blocked": the scales come from the quantisers' blocked outputs
    (utils.to_mx_grouped_blocked / to_mx_dim1_blocked) and the GEMMs take them
    in place; the e4m3 data and every result are the same bits."""
    import torch
    import utils

    random.seed(seed)
    gen = torch.Generator(device=device).manual_seed(seed)
    probs = []
    for (E, M, N, K) in shapes:
        offs = utils.generate_jagged_offs(E, M, multiple_of=multiple_of, device=device)
        A = torch.randn(M, K, device=device, dtype=torch.bfloat16, generator=gen)
        W = torch.randn(E, N, K, device=device, dtype=torch.bfloat16, generator=gen)
        G = torch.randn(M, N, device=device, dtype=torch.bfloat16, generator=gen)
        blk = scale_layout == "blocked"
        if "fwd" in passes:
            a_s, a_q = utils.to_mx_grouped_blocked(A, offs) if blk else utils.to_mx(A)
            b_s, b_q = utils.to_mx_grouped_blocked(W) if blk else utils.to_mx(W)
            probs.append(dict(pass_="fwd", shape=(E, M, N, K), flops=2.0 * M * N * K,
                              args=(a_q, b_q, a_s, b_s, offs), layout=scale_layout))
        if "fwd4" in passes:
            a_s, a_q = utils.to_mx(A)
            w4_s, w4_q = utils.to_mx(W, elem_dtype=torch.float4_e2m1fn_x2)
            probs.append(dict(pass_="fwd4", shape=(E, M, N, K), flops=2.0 * M * N * K,
                              args=(a_q, w4_q, a_s, w4_s, offs)))
        if "dgrad" in passes:
            if blk:
                g_s, g_q = utils.to_mx_grouped_blocked(G, offs)        # along N, per group
                wt_s, wt_q = utils.to_mx_grouped_blocked(W.transpose(-2, -1).contiguous())   # (E, K, N), per expert
            else:
                g_s, g_q = utils.to_mx(G)                              # along N
                wt = [utils.to_mx_dim1(W[e]) for e in range(E)]        # W[e]^T (K, N), along N
                wt_s = torch.stack([s for s, _ in wt])
                wt_q = torch.stack([q for _, q in wt])
            probs.append(dict(pass_="dgrad", shape=(E, M, N, K), flops=2.0 * M * N * K,
                              args=(g_q, wt_q, g_s, wt_s, offs), layout=scale_layout))
        if "wgrad" in passes:
            dim1 = utils.to_mx_dim1_blocked if blk else utils.to_mx_dim1
            go_s, go_q = dim1(G)                                       # (N, M), along tokens
            ia_s, ia_q = dim1(A)                                       # (K, M), along tokens
            probs.append(dict(pass_="wgrad", shape=(E, M, N, K), flops=2.0 * M * N * K,
                              args=(go_q, go_s, ia_q, ia_s, offs), layout=scale_layout))
        del A, W, G
    torch.cuda.synchronize()
    return probs


def build_ep_problems(device, shapes, passes, world, rank, seed=123, impl="fused"):
    """Expert-parallel sweep: the same 36 shapes with every rank holding its
    own M = 16640 tokens and the weights of the experts it hosts.  Group sizes
    are the single-GPU sweep's (same seed and draw order), rotated by rank so
    that every rank computes M rows.  fwd and dgrad
    run dispatch -> segment GEMM -> combine; wgrad runs on the hosting rank
    over the tokens it received (expert-major, as the forward's dispatch left
    them) and sums replicas' gradients (peer-memory replica sum, or an NCCL
    all-reduce for impl "nccl").  Per-rank FLOPs
    are 2*rows*N*K over the rows that rank computes; every rank sends all M of
    its rows, so the ranks' total is world * 2*M*N*K."""
    import torch
    import utils
    from mxgg import ep

    random.seed(seed)
    gen = torch.Generator(device=device).manual_seed(seed + 1000 * rank)
    probs = []
    groups = {}
    for (E, M, N, K) in shapes:
        pl = ep.ExpertPlacement(world, E)
        if E not in groups:
            groups[E] = ep.replica_groups(pl)          # collective: same order on every rank
        offs = utils.generate_jagged_offs(E, M, multiple_of=32, device="cpu").tolist()
        base = [b - a for a, b in zip([0] + offs[:-1], offs)]
        # every rank routes the same jagged distribution, rotated so that every
        # rank computes exactly M rows: the sweep measures dispatch, GEMM and
        # combine, not a router's load imbalance
        shift = (rank // pl.replicas) * pl.local
        counts = [base[(e - shift) % E] for e in range(E)]
        plan = ep.plan_dispatch(pl, counts, device)
        mine = pl.experts_of(rank)
        gw = torch.Generator(device=device).manual_seed(seed + 77 * (mine[0] + 1))
        Wl = torch.randn(len(mine), N, K, device=device, dtype=torch.bfloat16, generator=gw)
        if "fwd" in passes:
            A = torch.randn(M, K, device=device, dtype=torch.bfloat16, generator=gen)
            a_s, a_q = utils.to_mx(A)
            w_s, w_q = utils.to_mx(Wl)
            probs.append(dict(pass_="fwd", shape=(E, M, N, K), flops=2.0 * M * N * K, plan=plan, counts=counts,
                              args=(a_q, a_s), weights=(w_q, w_s)))
            del A
        if "dgrad" in passes:
            G = torch.randn(M, N, device=device, dtype=torch.bfloat16, generator=gen)
            g_s, g_q = utils.to_mx(G)
            wt = [utils.to_mx_dim1(Wl[e]) for e in range(len(mine))]
            probs.append(dict(pass_="dgrad", shape=(E, M, N, K), flops=2.0 * M * N * K, plan=plan, counts=counts,
                              args=(g_q, g_s), weights=(torch.stack([q for _, q in wt]),
                                                        torch.stack([s_ for s_, _ in wt]))))
            del G
        if "wgrad" in passes:
            R = plan.rows_recv
            loc = plan.expert_rows()
            loffs = torch.tensor(loc, dtype=torch.int64).cumsum(0).to(torch.int32).to(device)
            go = torch.randn(R, N, device=device, dtype=torch.bfloat16, generator=gen)
            x = torch.randn(R, K, device=device, dtype=torch.bfloat16, generator=gen)
            go_s, go_q = utils.to_mx_dim1(go)
            ia_s, ia_q = utils.to_mx_dim1(x)
            probs.append(dict(pass_="wgrad", shape=(E, M, N, K), flops=2.0 * M * N * K, plan=plan,
                              args=(go_q, go_s, ia_q, ia_s, loffs), groups=groups[E]))
            del go, x
        del Wl
    if impl == "fused" and any(p["pass_"] != "wgrad" for p in probs):
        # one set of shared buffers sized for the whole sweep
        import torch.distributed as dist
        cap = torch.tensor([max(p["plan"].rows_recv for p in probs)], device=device)
        dist.all_reduce(cap, op=dist.ReduceOp.MAX)
        kmax = max(max(s[2], s[3]) for s in shapes)
        fx = ep.FusedExpertParallel(ep.ExpertPlacement(world, world), int(cap.item()), M_TOKENS, kmax, kmax)
        for p in probs:
            if p["pass_"] != "wgrad":
                p["fused"] = (fx, fx.plan(p["counts"], ep.ExpertPlacement(world, p["shape"][0])))
    rep = [p for p in probs if p["pass_"] == "wgrad" and p["plan"].placement.replicas > 1]
    if impl == "fused" and rep:
        # replicated experts sum their weight gradients in place over peer memory
        nbytes = max(p["plan"].placement.local * p["shape"][2] * p["shape"][3] * 2 for p in rep)
        rs = ep.ReplicaSum(nbytes)
        for p in rep:
            p["rsum"] = rs
    torch.cuda.synchronize()
    return probs


MOE_TOKENS_PER_RANK = 16384
MOE_EXPERTS_PER_RANK = 8
MOE_D_MODEL, MOE_D_FF = 5120, 8192


def bench_moe(device, world, rank, steps, warmup):
    """BASELINE config 5, weak-scaled: 8 experts and 16384 tokens per rank
    (E = 64 and 131072 tokens at 8 GPUs), top-2 routing from seeded N(0,1)
    logits, up 5120 -> 8192 and down 8192 -> 5120, MXFP8 weights and MXFP4
    weights x MXFP8 activations.  One step = one layer forward over this
    rank's tokens (routing, quantise-on-dispatch, dispatch, both GEMMs,
    combine); TFLOPS counts the useful 2 * 2T * d_model * d_ff * 2 FLOPs of
    all ranks over the slowest rank's time."""
    import torch
    from mxgg import ep as ep_mod
    from mxgg.moe import MoELayer
    E = MOE_EXPERTS_PER_RANK * world
    T = MOE_TOKENS_PER_RANK
    g = torch.Generator(device=device).manual_seed(5 + rank)
    x = torch.randn(T, MOE_D_MODEL, device=device, dtype=torch.bfloat16, generator=g)
    logits = torch.randn(T, E, device=device, generator=g)
    placement = ep_mod.ExpertPlacement(world, E) if world > 1 else None
    fx = None
    if world > 1:
        cap = int(1.5 * 2 * T) + 32 * E
        fx = ep_mod.FusedExpertParallel(placement, max_recv_rows=cap, max_local_rows=2 * T + 32 * E,
                                        max_k=MOE_D_FF, max_n=MOE_D_FF)
    out = {"config": {"experts": E, "experts_per_gpu": MOE_EXPERTS_PER_RANK, "tokens": T * world,
                      "tokens_per_gpu": T, "top_k": 2, "d_model": MOE_D_MODEL, "d_ff": MOE_D_FF,
                      "routing": "softmax of seeded N(0,1) logits, top-2, renormalised; groups padded to 32"}}
    for name, fp4 in (("mxfp8", False), ("mxfp4_weights", True)):
        gw = torch.Generator(device=device).manual_seed(1000 + rank)
        up = torch.randn(MOE_EXPERTS_PER_RANK, MOE_D_FF, MOE_D_MODEL, device=device, dtype=torch.bfloat16,
                         generator=gw) * MOE_D_MODEL ** -0.5
        down = torch.randn(MOE_EXPERTS_PER_RANK, MOE_D_MODEL, MOE_D_FF, device=device, dtype=torch.bfloat16,
                           generator=gw) * MOE_D_FF ** -0.5
        layer = MoELayer(up, down, E, weights_fp4=fp4, placement=placement, ep=fx)
        del up, down
        for _ in range(warmup):
            layer.forward(x, logits)
        barrier(world)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(steps):
            layer.forward(x, logits)
        e.record()
        barrier(world)
        t = allreduce_max([s.elapsed_time(e) / steps * 1e-3], world)[0]
        out[name] = {"tflops": round(world * layer.flops(T) / t / 1e12, 1), "ms_per_step": round(t * 1e3, 3)}
        del layer
    if fx is not None:
        fx.close()
    return out


def run_ep_problem(p, marks=None):
    """One expert-parallel call; `marks` (3 events) split it into dispatch |
    local GEMM | combine."""
    import kernels
    from mxgg import ep
    from mxgg.ops import grouped_mm_segments
    plan = p["plan"]
    if p["pass_"] == "wgrad":
        if marks:
            marks[0].record()
        if "rsum" in p:
            # the gradient goes straight into this rank's peer-visible replica
            # buffer; on large grids the first part's replica sum overlaps the
            # second part's GEMM (the finish phase is then the second sum)
            from mxgg import tune
            go_q, _, ia_q, _, offs = p["args"]
            L, N, K = offs.shape[0], go_q.shape[0], ia_q.shape[0]
            out = p["rsum"].wgrad_sum(plan.placement, *p["args"], cfg=tune.call_config(tune.pick("wgrad", L, N, K)),
                                      gemm_done=marks[1] if marks else None)
        else:
            out = kernels.triton_mxfp8_wgrad(*p["args"])
            if marks:
                marks[1].record()
            ep.replica_allreduce(plan.placement, out, p.get("groups"))
        if marks:
            marks[2].record()
        return out
    if "fused" in p:
        # atom packing + copy issue | GEMM streaming over the arriving rows | barrier + inbox unpack
        fx, fplan = p["fused"]
        a_q, a_s = p["args"]
        w_q, w_s = p["weights"]
        fx.dispatch(fplan, a_q, a_s)
        if marks:
            marks[0].record()
        fx.gemm_received(fplan, a_q.shape[1], w_q, w_s, torch_bf16())
        if marks:
            marks[1].record()
        out = fx.finish(fplan, w_q.shape[1], torch_bf16())
        if marks:
            marks[2].record()
        return out
    recv_q, recv_s = ep.dispatch(plan, *p["args"])
    if marks:
        marks[0].record()
    y = grouped_mm_segments(recv_q, p["weights"][0], recv_s, p["weights"][1], plan.seg_offs, plan.seg_expert,
                               torch_bf16())
    if marks:
        marks[1].record()
    out = ep.combine(plan, y)
    if marks:
        marks[2].record()
    return out


def torch_bf16():
    import torch
    return torch.bfloat16


def ep_full_weights(device, pl, N, K, seed=123):
    """Every expert's (E, N, K) bf16 weights, regenerated from the seeds the
    hosting ranks drew them with in build_ep_problems."""
    import torch
    W = torch.empty(pl.n_experts, N, K, device=device, dtype=torch.bfloat16)
    done = set()
    for d in range(pl.world):
        mine = pl.experts_of(d)
        if mine[0] in done:
            continue                                   # a replica: same experts, same seed
        gw = torch.Generator(device=device).manual_seed(seed + 77 * (mine[0] + 1))
        W[mine[0]:mine[0] + len(mine)] = torch.randn(len(mine), N, K, device=device, dtype=torch.bfloat16,
                                                    generator=gw)
        done.update(mine)
    return W


def gpu_rel_l2(got, ref):
    import torch
    d = (got.double() - ref.double()).norm()
    n = ref.double().norm()
    return float(d / n) if float(n) > 0 else float(d)


def ep_parity(probs, world, rank, device, rel_tol=1e-3):
    """Check the expert-parallel outputs of this run against the single-GPU
    kernel (itself pinned to the oracle by the GPU tests) on the same
    rank-local operands: for every fwd / dgrad point, this rank's rows after
    dispatch -> streamed GEMM -> combine must match triton_mxfp8_grouped_mm of
    the rank's own tokens with every expert's weights, bit for bit where both
    deal the same tiles, else within rel-L2 `rel_tol` (bf16 outputs).  wgrad
    runs the single-GPU kernel on the hosting rank's own data, so it needs no
    separate check.  Returns this rank's per-point (rel_l2, exact) list."""
    import torch
    import kernels
    import utils
    out = []
    for p in probs:
        if p["pass_"] == "wgrad":
            continue
        E, M, N, K = p["shape"]
        pl = p["plan"].placement
        got = run_ep_problem(p).clone()
        offs = torch.tensor(p["counts"], dtype=torch.int64).cumsum(0).to(torch.int32).to(device)
        W = ep_full_weights(device, pl, N, K)
        if p["pass_"] == "fwd":
            w_s, w_q = utils.to_mx(W)
        else:
            wt = [utils.to_mx_dim1(W[e]) for e in range(E)]
            w_s = torch.stack([s_ for s_, _ in wt])
            w_q = torch.stack([q for _, q in wt])
        del W
        a_q, a_s = p["args"]
        ref = kernels.triton_mxfp8_grouped_mm(a_q, w_q, a_s, w_s, offs)
        rows = int(offs[-1].item()) if offs.numel() else 0
        g, r = got[:rows], ref[:rows]
        out.append((gpu_rel_l2(g, r), bool(torch.equal(g, r))))
        del w_q, w_s, ref, got
    torch.cuda.synchronize()
    return out


def moe_parity(device, world, rank, rel_tol=1e-3):
    """The expert-parallel MoE layer (config 5 shape, MXFP8 and MXFP4
    weights) against the single-GPU MoELayer holding every expert, on this
    rank's tokens.  Returns [(rel_l2, exact)] for the two weight formats."""
    import torch
    from mxgg import ep as ep_mod
    from mxgg.moe import MoELayer
    E = MOE_EXPERTS_PER_RANK * world
    T = MOE_TOKENS_PER_RANK
    g = torch.Generator(device=device).manual_seed(5 + rank)
    x = torch.randn(T, MOE_D_MODEL, device=device, dtype=torch.bfloat16, generator=g)
    logits = torch.randn(T, E, device=device, generator=g)
    placement = ep_mod.ExpertPlacement(world, E)
    fx = ep_mod.FusedExpertParallel(placement, max_recv_rows=int(1.5 * 2 * T) + 32 * E,
                                    max_local_rows=2 * T + 32 * E, max_k=MOE_D_FF, max_n=MOE_D_FF)
    res = []
    for fp4 in (False, True):
        ups, downs = [], []
        for d in range(world):
            gw = torch.Generator(device=device).manual_seed(1000 + d)
            ups.append(torch.randn(MOE_EXPERTS_PER_RANK, MOE_D_FF, MOE_D_MODEL, device=device, dtype=torch.bfloat16,
                                   generator=gw) * MOE_D_MODEL ** -0.5)
            downs.append(torch.randn(MOE_EXPERTS_PER_RANK, MOE_D_MODEL, MOE_D_FF, device=device,
                                     dtype=torch.bfloat16, generator=gw) * MOE_D_FF ** -0.5)
        sl = slice(rank * MOE_EXPERTS_PER_RANK, (rank + 1) * MOE_EXPERTS_PER_RANK)
        up_all, down_all = torch.cat(ups), torch.cat(downs)
        del ups, downs
        layer = MoELayer(up_all[sl].contiguous(), down_all[sl].contiguous(), E, weights_fp4=fp4,
                         placement=placement, ep=fx)
        y_ep = layer.forward(x, logits).clone()
        del layer
        ref = MoELayer(up_all, down_all, E, weights_fp4=fp4).forward(x, logits)
        res.append((gpu_rel_l2(y_ep, ref), bool(torch.equal(y_ep, ref))))
        del up_all, down_all, ref, y_ep
    fx.close()
    torch.cuda.synchronize()
    return res


def run_problem(p):
    import kernels
    if "plan" in p:
        return run_ep_problem(p)
    layout = p.get("layout", "row_major")
    if p["pass_"] == "wgrad":
        return kernels.triton_mxfp8_wgrad(*p["args"], scale_layout=layout)
    return kernels.triton_mxfp8_grouped_mm(*p["args"], scale_layout=layout)


def _blocked_scales(s2d):
    """(R, C) e8m0 scales -> the 128x4 blocked layout of block-scaled tensor
    cores (rows padded to 128, columns to 4; atom byte (r % 32) * 16 +
    (r % 128) // 32 * 4 + c % 4), returned as a (R', C') tensor."""
    import torch
    R, C = s2d.shape
    Rp, Cp = -(-R // 128) * 128, -(-C // 4) * 4
    pad = torch.zeros((Rp, Cp), dtype=torch.uint8, device=s2d.device)
    pad[:R, :C] = s2d.view(torch.uint8)
    b = pad.view(Rp // 128, 128, Cp // 4, 4).permute(0, 2, 1, 3).reshape(-1, 4, 32, 4).transpose(1, 2)
    return b.reshape(Rp, Cp)


def torch_grouped_arm(device, shapes, steps=5):
    """torch's own MXFP8 grouped GEMM (torch._scaled_grouped_mm, sm_100) on
    the same forward points, beside this library's: its counterpart of the
    reference's vendor comparison arms (bench.py:95-110).  Scales are re-laid
    into torch's per-group blocked layout outside the timed region (this
    library packs its own scales inside every call).  Returns per-point
    TFLOPS and the rel-L2 between the two outputs, or why torch refused."""
    import random

    import torch

    import kernels
    import utils
    rows = []
    for (E, M, N, K) in shapes:
        random.seed(123)
        g = torch.Generator(device=device).manual_seed(123)
        offs = utils.generate_jagged_offs(E, M, multiple_of=32, device=device)
        A = torch.randn(M, K, device=device, dtype=torch.bfloat16, generator=g)
        W = torch.randn(E, N, K, device=device, dtype=torch.bfloat16, generator=g)
        a_s, a_q = utils.to_mx(A)
        b_s, b_q = utils.to_mx(W)
        ends = [0] + offs.tolist()
        sa = torch.cat([_blocked_scales(a_s[ends[i]:ends[i + 1]]) for i in range(E) if ends[i + 1] > ends[i]])
        sb = torch.stack([_blocked_scales(b_s[e]).reshape(-1) for e in range(E)])   # (E, blocked N x K/32)
        sa, sb = sa.view(torch.float8_e8m0fnu), sb.view(torch.float8_e8m0fnu)
        ours = kernels.triton_mxfp8_grouped_mm(a_q, b_q, a_s, b_s, offs)
        try:
            theirs = torch._scaled_grouped_mm(a_q, b_q.transpose(-2, -1), sa, sb, offs=offs,
                                              out_dtype=torch.bfloat16)
        except Exception as e:   # torch rejects the layout or has no sm_100 MXFP8 grouped path
            return {"unavailable": f"{type(e).__name__}: {str(e).splitlines()[0][:200]}"}
        torch.cuda.synchronize()
        d = (theirs.float() - ours.float()).norm() / ours.float().norm().clamp_min(1e-30)

        def t(fn):
            for _ in range(2):
                fn()
            ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
            scratch = torch.empty(512 << 20, dtype=torch.uint8, device=device)
            for s_, e_ in ev:
                scratch.zero_()
                s_.record()
                fn()
                e_.record()
            torch.cuda.synchronize()
            return sum(s_.elapsed_time(e_) for s_, e_ in ev) / steps * 1e-3

        fl = 2.0 * M * N * K
        t_ours = t(lambda: kernels.triton_mxfp8_grouped_mm(a_q, b_q, a_s, b_s, offs))
        t_theirs = t(lambda: torch._scaled_grouped_mm(a_q, b_q.transpose(-2, -1), sa, sb, offs=offs,
                                                      out_dtype=torch.bfloat16))
        # the reference bench's own baseline column: bf16 torch._grouped_mm (bench.py:125-183)
        t_bf16 = t(lambda: torch._grouped_mm(A, W.transpose(-2, -1), offs=offs))
        rows.append({"E": E, "N": N, "K": K, "mxgg_tflops": round(fl / t_ours / 1e12, 1),
                     "torch_tflops": round(fl / t_theirs / 1e12, 1), "bf16_tflops": round(fl / t_bf16 / 1e12, 1),
                     "rel_l2": float(f"{d.item():.3g}")})
        del a_q, b_q, a_s, b_s, sa, sb, ours, theirs, A, W
    return {"points": rows,
            "mxgg_geomean": round(geomean([r["mxgg_tflops"] for r in rows]), 1),
            "torch_geomean": round(geomean([r["torch_tflops"] for r in rows]), 1),
            "bf16_grouped_mm_geomean": round(geomean([r["bf16_tflops"] for r in rows]), 1),
            "note": "forward calls; torch's scale re-layout is outside its timed region; bf16 = "
                    "torch._grouped_mm on the unquantised operands (the reference bench's baseline)"}


def vendor_arm(probs, steps, flush):
    """torch's own sm_100 MXFP8 grouped GEMM (torch._scaled_grouped_mm) on
    every forward point of this run, timed exactly as this library's calls
    are (one CUDA graph per call, L2 flushed before each timed replay, CUDA
    events), with its per-group 128x4 blocked scales prepared outside the
    timed region.  Returns its geomean and ours on the same points."""
    import torch
    fwd = [p for p in probs if p["pass_"] == "fwd"]
    if not fwd:
        return None
    fns = []
    for p in fwd:
        a_q, b_q, a_s, b_s, offs = p["args"]
        E = b_q.shape[0]
        ends = [0] + offs.tolist()
        sa = torch.cat([_blocked_scales(a_s[ends[i]:ends[i + 1]]) for i in range(E) if ends[i + 1] > ends[i]])
        sb = torch.stack([_blocked_scales(b_s[e]).reshape(-1) for e in range(E)])
        sa, sb = sa.view(torch.float8_e8m0fnu), sb.view(torch.float8_e8m0fnu)
        fns.append((lambda a_q=a_q, b_q=b_q, sa=sa, sb=sb, offs=offs:
                    torch._scaled_grouped_mm(a_q, b_q.transpose(-2, -1), sa, sb, offs=offs,
                                             out_dtype=torch.bfloat16)))
    try:
        fns[0]()
        torch.cuda.synchronize()
    except Exception as e:   # no sm_100 MXFP8 grouped path in this torch build
        return {"unavailable": f"{type(e).__name__}: {str(e).splitlines()[0][:200]}"}
    graphs, keep = [], []
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for fn in fns:
            fn()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=side):
                keep.append(fn())
            graphs.append(g)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    per = []
    for g in graphs:
        ts = []
        for it in range(steps + 2):
            flush()
            s_, e_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s_.record()
            g.replay()
            e_.record()
            e_.synchronize()
            if it >= 2:
                ts.append(s_.elapsed_time(e_) * 1e-3)
        per.append(sum(ts) / len(ts))
    tf = [p["flops"] / t / 1e12 for p, t in zip(fwd, per)]
    return {"kernel": "torch._scaled_grouped_mm (MXFP8, sm_100)", "points": len(fwd),
            "fwd_geomean_tflops": round(geomean(tf), 1),
            "per_point_tflops": [round(x, 1) for x in tf],
            "timing": "one CUDA graph per call, L2 flushed before every timed replay, as this library's line"}


# ------------------------------------------------------------------ peaks
def measured_mxfp8_ceiling(device):
    """cuBLAS MXFP8 dense GEMM (torch._scaled_mm, 8192^3, e8m0 1x32 scales),
    best of 10 -- the MXFP8 tensor ceiling of this GPU in this run."""
    import torch
    import utils
    try:
        n = 8192
        a = torch.randn(n, n, device=device, dtype=torch.bfloat16)
        b = torch.randn(n, n, device=device, dtype=torch.bfloat16)
        sa, qa = utils.to_mx_blocked_scales(a)
        sb, qb = utils.to_mx_blocked_scales(b)
        sa = sa.view(torch.float8_e8m0fnu)
        sb = sb.view(torch.float8_e8m0fnu)
        fn = lambda: torch._scaled_mm(qa, qb.t(), scale_a=sa, scale_b=sb, out_dtype=torch.bfloat16)  # noqa: E731
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        best = float("inf")
        for _ in range(10):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            fn()
            e.record()
            torch.cuda.synchronize()
            best = min(best, s.elapsed_time(e) * 1e-3)
        return {"tflops": round(2 * n ** 3 / best / 1e12, 1), "how": "torch._scaled_mm MXFP8 8192^3, best of 10"}
    except Exception as exc:  # pragma: no cover - reported, not fatal
        return {"tflops": None, "how": f"torch._scaled_mm MXFP8 unavailable: {type(exc).__name__}: {exc}"[:200]}


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


def load_traffic():
    path = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f)
    return {}


# ------------------------------------------------------------------ CPU arm
def cpu_path_sample(threads):
    """The reference's CPU path (to_mx + dequantise + per-group fp32 torch
    matmul, oracle/cpu_path.py) over a bounded sample of the sweep."""
    from oracle.cpu_path import CpuPathSample
    return CpuPathSample(threads=threads)


def gpu_smi_id(dev):
    """nvidia-smi -i accepts the GPU UUID, which survives CUDA_VISIBLE_DEVICES remapping."""
    import torch
    try:
        return "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        return str(dev.index or 0)


def quantize_bandwidth(dev, hbm_gbs):
    """to_mx over a full sweep operand (16640 x 8192 bf16), L2 flushed, median of 20."""
    import torch
    import utils
    x = torch.randn(M_TOKENS, 8192, device=dev, dtype=torch.bfloat16)
    for _ in range(3):
        utils.to_mx(x)
    ts = []
    for _ in range(20):
        utils.flush_l2(dev)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        utils.to_mx(x)
        e.record()
        torch.cuda.synchronize()
        ts.append(s.elapsed_time(e) * 1e-3)
    t = sorted(ts)[len(ts) // 2]
    nbytes = x.numel() * 2 + x.numel() + x.numel() // 32
    gbs = nbytes / t / 1e9
    return {"bound": "hbm", "kernel": "mxgg::quantize_rows_e4m3", "achieved": round(gbs, 1), "peak": hbm_gbs,
            "unit": "GB/s", "frac": round(gbs / hbm_gbs, 4), "us": round(t * 1e6, 1),
            "algorithmic_bytes": nbytes}


def cpu_cores():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count()


# ------------------------------------------------------------------ main arms
def dist_setup(args):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        # no NVLink multicast objects: a rank that dies while bound to one can
        # fault its peers' GPUs; plain NVLink transfers are what we time
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    import torch
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()


def allreduce_max(vals, world):
    import torch
    if world == 1:
        return vals
    import torch.distributed as dist
    t = torch.tensor(vals, dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def capture_graphs(probs):
    """One CUDA graph per problem (its scale pack + GEMM launches): replaying
    it keeps host launch overhead out of the device timing."""
    import torch
    graphs = []
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for p in probs:
            run_problem(p)                    # warm: first-use setup outside the capture
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=side):
                p["graph_out"] = run_problem(p)
            graphs.append(g)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    return graphs


def time_ep_problems(probs, steps, warmup, world, flush):
    """Expert-parallel sweep, eager (NCCL calls are not captured): per-problem
    mean device time (s) and per-phase times (dispatch, GEMM, combine)."""
    import torch
    n = len(probs)
    for _ in range(warmup):
        for p in probs:
            flush()
            run_ep_problem(p)
    barrier(world)
    ev = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731
    rec = [[(ev(), ev(), ev(), ev(), ev()) for _ in range(n)] for _ in range(steps)]
    step_s, step_e = ev(), ev()
    step_s.record()
    for s in range(steps):
        for i, p in enumerate(probs):
            flush()
            e = rec[s][i]
            e[0].record()
            run_ep_problem(p, marks=e[1:4])
            e[4].record()
    step_e.record()
    barrier(world)
    per = [sum(rec[s][i][0].elapsed_time(rec[s][i][4]) for s in range(steps)) / steps * 1e-3 for i in range(n)]
    phases = [[sum(rec[s][i][k].elapsed_time(rec[s][i][k + 1]) for s in range(steps)) / steps * 1e-3
               for k in range(3)] for i in range(n)]
    return per, phases, step_s.elapsed_time(step_e) / steps


def time_problems(probs, steps, warmup, world, flush):
    """Per-problem mean device time (s) over `steps` timed steps."""
    import torch
    n = len(probs)
    graphs = capture_graphs(probs)
    for _ in range(warmup):
        for g in graphs:
            flush()
            g.replay()
    barrier(world)
    starts = [[torch.cuda.Event(enable_timing=True) for _ in range(n)] for _ in range(steps)]
    ends = [[torch.cuda.Event(enable_timing=True) for _ in range(n)] for _ in range(steps)]
    barrier(world)
    step_s = torch.cuda.Event(enable_timing=True)
    step_e = torch.cuda.Event(enable_timing=True)
    step_s.record()
    for s in range(steps):
        for i, g in enumerate(graphs):
            flush()
            starts[s][i].record()
            g.replay()
            ends[s][i].record()
    step_e.record()
    barrier(world)
    per = [sum(starts[s][i].elapsed_time(ends[s][i]) for s in range(steps)) / steps * 1e-3 for i in range(n)]
    wall_ms = step_s.elapsed_time(step_e) / steps
    del graphs
    for p in probs:
        p.pop("graph_out", None)
    return per, wall_ms


def time_e2e(probs, steps, warmup, world):
    """Same sweep through the public API with pinned host inputs/outputs.

    One GPU: each call goes through ``mxgg.host.HostPipeline`` (the call cut
    into pieces on three streams, so the copies in and out overlap the
    GEMMs); the events bracket the whole call, first copy in to last copy
    out.  Expert parallel (N > 1): the rank's inputs are copied in, the call
    runs, its output is copied out, one after another."""
    import torch
    pipe = None
    if world == 1:
        from mxgg.host import HostPipeline
        pipe = HostPipeline(pieces=8)
    max_in = max(sum(t.numel() * t.element_size() for t in p["args"]) for p in probs)
    host_in = torch.empty(max_in + 4096 * 8, dtype=torch.uint8, pin_memory=True)
    per = []
    h2d_total, d2h_total = 0, 0
    for p in probs:
        # stage this problem's inputs in pinned host memory (untimed)
        host_views, off = [], 0
        for t in p["args"]:
            nb = t.numel() * t.element_size()
            hv = host_in[off:off + nb]
            hv.copy_(t.contiguous().view(torch.uint8).reshape(-1))
            host_views.append((hv, t.shape, t.dtype))
            off += (nb + 511) // 512 * 512
        out_like = run_problem(p)
        host_out = torch.empty(out_like.shape, dtype=out_like.dtype, pin_memory=True)
        del out_like
        if pipe is not None:
            hosts = [hv.view(dt).view(shape) for (hv, shape, dt) in host_views]
            ends = p["args"][4].tolist()                  # the offsets travel inside the call (pinned table)

            def call():
                if p["pass_"] == "wgrad":
                    pipe.wgrad(*hosts[:4], ends, host_out)
                else:
                    pipe.grouped_mm(*hosts[:4], ends, host_out, host_out.dtype)
        else:
            dev_args = [torch.empty(shape, dtype=dt, device="cuda") for (_, shape, dt) in host_views]
            q = dict(p)
            q["args"] = tuple(dev_args)

            def call():
                for (hv, shape, dt), d in zip(host_views, dev_args):
                    d.view(torch.uint8).reshape(-1).copy_(hv, non_blocking=True)
                out = run_problem(q)
                host_out.copy_(out, non_blocking=True)
        ts = []
        for it in range(warmup + steps):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            call()
            e.record()
            torch.cuda.synchronize()
            if it >= warmup:
                ts.append(s.elapsed_time(e) * 1e-3)
        per.append(sum(ts) / len(ts))
        h2d_total += sum(hv.numel() for hv, _, _ in host_views)
        d2h_total += host_out.numel() * host_out.element_size()
        del host_out
    per = allreduce_max(per, world)
    return per, h2d_total, d2h_total


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="mxgg", choices=["mxgg", "reference"])
    ap.add_argument("--passes", default="fwd,dgrad,wgrad")
    ap.add_argument("--shapes", default="all", help="'all' or comma list of shape indices 0..35")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip e2e, the CPU sample, the cuBLAS ceiling and the quantiser line (profiling runs)")
    ap.add_argument("--detail", action="store_true", help="also print one JSON line per (shape, pass) to stderr")
    ap.add_argument("--tile-m", type=int, default=0, help="GEMM tile rows: 128 (one CTA) or 256 (CTA pair); 0 = auto")
    ap.add_argument("--tile-n", type=int, default=0, help="GEMM tile columns: 128 or 256; 0 = auto")
    ap.add_argument("--schedule", default="default", choices=["default", "tiles", "split_tail"],
                    help="GEMM work schedule: deal whole tiles (tiles, the default) or split the last "
                         "partial round's tiles along the contraction (split_tail)")
    ap.add_argument("--split-max", type=int, default=0, help="most pieces per split tile (0 = automatic)")
    ap.add_argument("--torch-arm", action="store_true",
                    help="also time torch._scaled_grouped_mm (MXFP8) on the same forward shapes (1 GPU)")
    ap.add_argument("--ep-impl", default="fused", choices=["fused", "nccl"],
                    help="N > 1: peer-memory dispatch with the combine fused into the GEMM (fused), "
                         "or NCCL all-to-all dispatch/combine around the segment GEMM (nccl)")
    args = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    passes = [p for p in args.passes.split(",") if p]
    shapes = llama4_shapes()
    idx = list(range(36)) if args.shapes == "all" else [int(i) for i in args.shapes.split(",")]
    cfg = {"workload": "llama4-36-shapes x {" + ",".join(passes) + "}", "shapes": len(idx), "M": M_TOKENS,
           "tile": f"{args.tile_m or 'auto'}x{args.tile_n or 'auto'}",
           "E": [1, 2, 4, 8], "N": [2048, 5120, 8192], "K": [2048, 5120, 8192], "offs": "generate_jagged_offs(seed 123, multiple_of 32)",
           "l2": "flushed (512 MiB memset) before every timed launch", "parallelism": "single GPU"}

    if args.impl == "reference":
        # The reference's GEMM kernels are Triton for gfx950 only and cannot
        # run on this machine; its runnable path is the CPU one: to_mx,
        # dequantise, per-group fp32 matmul (oracle/cpu_path.py), timed on
        # this host's cores.  Each step is one (shape, pass) point of a
        # 12-point sample at the sweep's full M, taken in turn.
        if rank != 0:
            return 0
        threads = cpu_cores()
        ref = cpu_path_sample(threads)
        vals = []
        for it in range(args.warmup + args.steps):
            v = ref.run_point(it)
            if it >= args.warmup:
                vals.append(v)
        v = geomean(vals)
        sample_cfg = {"workload": "reference CPU path on a sample of the llama4 sweep",
                      "points": [f"{p[0]} E={p[1][0]} N={p[1][1]} K={p[1][2]}" for p in ref.points],
                      "M": ref.M, "offs": "generate_jagged_offs draw (seed 123, multiple_of 32)",
                      "steps_cover": "one point per step, in turn"}
        line = {"metric": METRIC, "value": round(v, 4), "unit": "TFLOPS", "impl": "reference", "n_gpus": args.gpus,
                "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "e4m3xe4m3->f32", "data": "synthetic", "config": sample_cfg,
                "cpu_baseline": {"value": round(v, 4), "unit": "TFLOPS", "cores": threads, "kind": "port",
                                 "sample": ref.describe()},
                "e2e": {"value": round(v, 4), "unit": "TFLOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return 0

    import torch
    world, rank, local = dist_setup(args)
    import mxgg
    import utils
    dev = torch.device("cuda", torch.cuda.current_device())
    mxgg.device_status(clear=True)
    if args.tile_m or args.tile_n or args.schedule != "default" or args.split_max:
        # an explicit configuration on the command line wins over the packaged tuned table
        from mxgg import tune as _tune
        _tune.install(None)
    mxgg.set_tile_config(args.tile_m, args.tile_n, 0)
    mxgg.set_schedule({"default": mxgg._lib.SCHED_DEFAULT, "tiles": mxgg._lib.SCHED_TILES,
                       "split_tail": mxgg._lib.SCHED_SPLIT_TAIL}[args.schedule], args.split_max)

    ep_mode = world > 1
    if ep_mode:
        probs = build_ep_problems(dev, [shapes[i] for i in idx], passes, world, rank, impl=args.ep_impl)
        cfg["parallelism"] = (f"ep{world} (expert parallel: peer-memory dispatch, combine fused into the GEMM "
                              "epilogue over NVLink)" if args.ep_impl == "fused" else
                              f"ep{world} (expert parallel: NCCL all-to-all dispatch/combine)")
        cfg["M"] = f"{M_TOKENS} tokens per rank"
    else:
        probs = build_problems(dev, [shapes[i] for i in idx], passes)
    utils.flush_l2(dev)
    flush = lambda: utils.flush_l2(dev)  # noqa: E731

    phases = None
    with ClockSampler(gpu_smi_id(dev)) as clk:
        # a short untimed pre-run keeps the sampler's window on a loaded GPU
        for p_ in probs[: min(len(probs), 12)]:
            flush()
            run_problem(p_)
        if ep_mode:
            per, phases, wall_ms = time_ep_problems(probs, args.steps, args.warmup, world, flush)
        else:
            per, wall_ms = time_problems(probs, args.steps, args.warmup, world, flush)
    per = allreduce_max(per, world)
    status = mxgg.device_status(clear=True)
    ep_info = None
    if ep_mode:
        # rank 0's own GEMM work and phase split (max over ranks per phase)
        ph = allreduce_max([x for row in phases for x in row], world)
        phases = [ph[3 * i:3 * i + 3] for i in range(len(probs))]
        # rows each timed GEMM phase multiplies: the received rows (fused: peers' rows only)
        local_flops = [2.0 * (p["fused"][1].rows_recv if "fused" in p else p["plan"].rows_recv)
                       * p["shape"][2] * p["shape"][3] for p in probs]
        gemm_t = [x[1] for x in phases]
        ep_info = {"phases_us_per_step": {
                       "dispatch_issue": round(1e6 * sum(x[0] for p, x in zip(probs, phases)
                                                         if p["pass_"] != "wgrad"), 1),
                       "streamed_gemm_or_wgrad": round(1e6 * sum(gemm_t), 1),
                       "finish_or_replica_allreduce": round(1e6 * sum(x[2] for x in phases), 1)},
                   "rank0_gemm_tflops_geomean": round(geomean([f / t / 1e12 for f, t in zip(local_flops, gemm_t)]), 1),
                   "placement": "experts sharded when E >= world, replicated (world/E copies) when E < world"}

    tf = [p["flops"] / t / 1e12 for p, t in zip(probs, per)]
    by_pass = {ps: round(geomean([x for x, p in zip(tf, probs) if p["pass_"] == ps]), 1) for ps in passes}
    gm = geomean(tf)
    total_flops = sum(p["flops"] for p in probs)
    total_time = sum(per)
    achieved = total_flops / total_time / 1e12
    if ep_mode:
        # the GEMM kernel's own rate on rank 0 (communication excluded)
        achieved = sum(local_flops) / sum(gemm_t) / 1e12

    e2e = None
    if args.no_extras:
        args.no_e2e = args.no_cpu = True
    if not args.no_e2e:
        per_e, h2d, d2h = time_e2e(probs, max(1, args.steps), max(1, min(args.warmup, 2)), world)
        e2e = {"value": round(world * geomean([p["flops"] / t / 1e12 for p, t in zip(probs, per_e)]), 1),
               "unit": "TFLOPS", "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
               "path": ("mxgg.host.HostPipeline: 8 pieces, copies in / GEMMs / copies out on 3 streams"
                        if world == 1 else "copy in, expert-parallel call, copy out")}

    if rank == 0 and args.detail:
        for i, (p, t) in enumerate(zip(probs, per)):
            row = {"pass": p["pass_"], "shape": p["shape"], "us": round(t * 1e6, 1),
                   "tflops": round(p["flops"] / t / 1e12, 1)}
            if phases is not None:
                row["phases_us"] = [round(x * 1e6, 1) for x in phases[i]]
            print(json.dumps(row), file=sys.stderr)

    ceiling = measured_mxfp8_ceiling(dev) if rank == 0 and not args.no_extras else None
    peaks, peaks_src = load_peaks()
    traffic = load_traffic()
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        ref = cpu_path_sample(cpu_cores())
        ref.run_point(0)                      # warm-up (thread pool, allocator)
        cpu = {"value": round(geomean([ref.run_point(i) for i in range(len(ref.points))]), 4), "unit": "TFLOPS",
               "cores": ref.threads, "kind": "port", "sample": ref.describe()}
    quant = quantize_bandwidth(dev, peaks.get("hbm_gbs", 6650.0)) if rank == 0 and not args.no_extras else None
    n_main = len(probs)
    moe = None if args.no_extras else bench_moe(dev, world, rank, max(2, min(args.steps, 5)), 2)
    vendor = None
    if world == 1 and not args.no_extras:
        vendor = vendor_arm(probs, max(3, min(args.steps, 5)), flush)
        if vendor and "fwd_geomean_tflops" in vendor and "fwd" in by_pass:
            vendor["mxgg_fwd_geomean_tflops"] = by_pass["fwd"]
            vendor["mxgg_over_vendor"] = round(by_pass["fwd"] / vendor["fwd_geomean_tflops"], 3)
    fp4 = None
    if world == 1 and not args.no_extras:
        # MXFP4 weights x MXFP8 activations, the same 36 forward shapes
        n_main = len(probs)
        del probs
        probs = []
        p4 = build_problems(dev, [shapes[i] for i in idx], ["fwd4"])
        per4, _ = time_problems(p4, max(1, min(args.steps, 3)), 1, world, flush)
        fp4 = {"fwd_geomean_tflops": round(geomean([p["flops"] / t / 1e12 for p, t in zip(p4, per4)]), 1),
               "note": "e2m1 weights (two per byte, TMA-unpacked) x e4m3 activations on kind::mxf8f6f4"}
        del p4
    blocked = None
    if world == 1 and not args.no_extras:
        # the same sweep with the scales quantised straight into the blocked
        # layout the GEMM reads (no pack launch per call)
        pb = build_problems(dev, [shapes[i] for i in idx], passes, scale_layout="blocked")
        perb, _ = time_problems(pb, max(1, min(args.steps, 3)), 1, world, flush)
        tfb = [p["flops"] / t / 1e12 for p, t in zip(pb, perb)]
        blocked = {"geomean_tflops": round(geomean(tfb), 1),
                   "per_pass_geomean": {ps: round(geomean([x for x, p in zip(tfb, pb) if p["pass_"] == ps]), 1)
                                        for ps in passes},
                   "over_row_major": round(geomean(tfb) / gm, 4),
                   "launches_per_call": 1,
                   "scales": "utils.to_mx_grouped_blocked / to_mx_dim1_blocked outside the timed region; "
                             "scale_layout='blocked'"}
        del pb
    mult16 = None
    if world == 1 and not args.no_extras and any(ps in passes for ps in ("fwd", "dgrad")):
        # BASELINE config 2's group sizes: multiples of 16 (fwd and dgrad;
        # wgrad's token blocks need 32, as in the reference)
        p16 = build_problems(dev, [shapes[i] for i in idx], [ps for ps in passes if ps in ("fwd", "dgrad")],
                             multiple_of=16)
        per16, _ = time_problems(p16, max(1, min(args.steps, 3)), 1, world, flush)
        tf16 = [p["flops"] / t / 1e12 for p, t in zip(p16, per16)]
        mult16 = {"fwd_dgrad_geomean_tflops": round(geomean(tf16), 1),
                  "per_pass_geomean": {ps: round(geomean([x for x, p in zip(tf16, p16) if p["pass_"] == ps]), 1)
                                       for ps in ("fwd", "dgrad") if ps in passes},
                  "offs": "generate_jagged_offs(seed 123, multiple_of 16)"}
        del p16

    parity = None
    if ep_mode:
        # after the timed region: every rank checks its own rows against the
        # single-GPU kernel; the worst rank decides
        pts = ep_parity(probs, world, rank, dev)
        if not args.no_extras:
            pts += moe_parity(dev, world, rank)
        worst = allreduce_max([x[0] for x in pts], world)
        exact = allreduce_max([0.0 if x[1] else 1.0 for x in pts], world)
        st_after = mxgg.device_status(clear=True)
        st_all = allreduce_max([float(st_after)], world)[0]
        parity = {"points": len(pts), "max_rel_l2": max(worst) if worst else 0.0,
                  "bit_exact_points": sum(1 for v in exact if v == 0.0), "tolerance": 1e-3,
                  "device_status": int(st_all),
                  "against": "triton_mxfp8_grouped_mm on one GPU, same rank-local operands, every expert's "
                             "weights (fwd and dgrad points)" + ("" if args.no_extras else
                                                                 "; MoE layer vs single-GPU MoELayer (2 points)")}
    if rank == 0:
        # MXFP8 ceiling: 2 x the measured dense bf16 rate (sm_100 runs
        # kind::mxf8f6f4 at twice kind::f16's rate per SM)
        peak = round(2.0 * peaks.get("bf16_tflops", 1590.0), 1)
        roof = {"bound": "tensor", "kernel": "mxgg::grouped_gemm_kernel", "achieved": round(achieved, 1),
                "peak": peak, "unit": "TFLOP/s", "frac": round(achieved / peak, 4),
                "peak_source": f"2 x bf16_tflops of {peaks_src} (measured cuBLAS bf16 burst; MXFP8 runs at twice "
                               "the bf16 tensor rate)",
                "frac_of_nominal_4500": round(achieved / NOMINAL_MXFP8_TFLOPS, 4),
                "cublas_mxfp8_8192cube": ceiling,
                "traffic": traffic.get("grouped_gemm_bytes_per_launch")}
        line = {"metric": METRIC, "value": round(world * gm, 1), "unit": "TFLOPS", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(total_time * 1e3, 3),
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "e4m3xe4m3->f32 (bf16 out)", "data": "synthetic", "config": cfg,
                "per_pass_geomean": by_pass, "pct_of_nominal_peak": round(100 * gm / NOMINAL_MXFP8_TFLOPS, 2),
                "pct_of_measured_mxfp8": round(100 * gm / peak, 2),
                "roofline": roof, "quantize_roofline": quant, "cpu_baseline": cpu, "e2e": e2e,
                "gpu_launches": 2 * n_main * args.steps, "clocks": clk.summary(),
                "device_status": status, "wall_ms_per_step": round(wall_ms, 3)}
        if ep_info:
            line["expert_parallel"] = ep_info
        if parity is not None:
            line["ep_parity"] = parity
        if moe:
            line["moe_layer"] = moe
        if fp4:
            line["mxfp4_weights"] = fp4
        if mult16:
            line["fwd_dgrad_mult16"] = mult16
        if blocked:
            line["blocked_scales"] = blocked
        if vendor:
            line["vs_vendor"] = vendor
        if args.torch_arm and world == 1:
            line["torch_scaled_grouped_mm"] = torch_grouped_arm(dev, [shapes[i] for i in idx])
        print(json.dumps(line), flush=True)
    if world > 1:
        barrier(world)
        for fx in {id(p["fused"][0]): p["fused"][0] for p in probs if "fused" in p}.values():
            fx.close()
        for rs in {id(p["rsum"]): p["rsum"] for p in probs if "rsum" in p}.values():
            rs.close()
        import torch.distributed as dist
        dist.destroy_process_group()
    if parity is not None and (parity["max_rel_l2"] > parity["tolerance"] or parity["device_status"] != 0):
        print(f"expert-parallel parity failed: {parity}", file=sys.stderr)
        return 3
    return 0


if __name__ == "__main__":
    sys.exit(main())
