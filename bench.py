#!/usr/bin/env python
"""Benchmark of the H3 DiT hot path on B200 (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload dit_block|dit_step|linear|fused|a2a|qkv_a2a|quant|gemm|vs_triton|nvlink_probe]
                    [--seq S] [--exchange p2p|nccl] [--overlap G] [--rows M] [--cols K] [--act none|gelu]
                    [--blocks B] [--convrot 64|256] [--qknorm] [--peers P]
                    [--no-cpu-baseline] [--no-e2e] [--no-parity] [--no-step] [--no-a2a]

Default workload (dit_block): one synthetic DiT block of the benchmark's
block configuration -- D=5120, 40 heads x 128, FFN 13824 (GELU-tanh), four
INT8 linears with per-channel scales + bias, the fused adaLN norm / gate
chain, Ulysses all-to-all around SDPA over S=128000 tokens -- split over N
GPUs by sequence (strong scaling).  A step is one block forward over the
rank's rows (the residual stream is restored from the step's input first).
Timing: W untimed steps, then K steps between barrier + synchronize, CUDA
events on the compute stream, max over ranks.  Inputs (x 1.31 GB/N, weights
245 MB) exceed the 126 MB L2, so no flush is needed between steps.

Prints ONE JSON line on rank 0.  `value` is ms per step (lower is better);
`e2e` repeats the step through host buffers (pinned H2D of the step's input
rows and conditioning, D2H of the output rows, every step inside the timed
region) with h3b.model.HostPipeline, whose copy streams move step k+1's input
and step k-1's output during step k; `e2e.serial_ms_per_step` is the same with
copies and compute in sequence on one stream; `roofline` is the INT8 GEMM
(the dominant kernel of this library) timed by CUDA events inside the timed
region; `cpu_baseline` times the reference's eager PyTorch path on the host's
cores on a bounded sample of the same workload (rank 0, N=1 only).
`--impl reference` prints the CPU reference path's line instead (rank 0 only).
After every timed region a checker leg compares the timed path's output with
the reference's eager path on the same rows (`parity`, bit for bit, summed over
ranks; at N > 1 the eager exchange is all_to_all_single over NCCL).  The
default line also carries `dit_step` (configuration 4: 40 blocks, S=252000,
512 text tokens; one block forward of warm-up, 2 timed steps, 1 step end to
end, and the final latent's parity) and, at N > 1, `a2a` (configuration 2 on
both exchange back ends, bus GB/s, an identity round trip checked bit for bit,
NVML's NVLink byte counters around the timed region).
The other workloads are for measurements by hand: linear = single INT8 linear
of config 0, fused = the fused chain of config 1, a2a = the Ulysses exchange of
config 2, dit_step = the 40-block step alone, qkv_a2a = one rank's qkv GEMM with
the forward exchange in its epilogue (the ranks' buffers emulated on one GPU),
quant = the activation quantiser (--act gelu: the GELU quantiser), gemm = the
block's four GEMM shapes, vs_triton = the reference's own Triton kernels against
this library's on the same GPU, nvlink_probe = one process driving two GPUs
through the forward exchange (for ncu's NVLink counters).
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from datetime import timedelta

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (ROOT, os.path.join(ROOT, "minimax-h3-multi-dgx-spark_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

PEAKS_FILE = os.path.join(ROOT, "MEASURED_PEAKS.json")
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["dit_block", "dit_step", "linear", "fused", "a2a", "qkv_a2a", "quant",
                                           "vs_triton", "nvlink_probe", "gemm"],
                    default="dit_block")
    ap.add_argument("--peers", type=int, default=8, help="ranks emulated by the qkv_a2a workload")
    ap.add_argument("--qknorm", action="store_true", help="qkv_a2a workload: with the per-head q/k RMSNorm")
    ap.add_argument("--convrot", type=int, default=0, choices=[0, 64, 256],
                    help="linear workload: ConvRot quantiser with this rotation group (0 = plain)")
    ap.add_argument("--seq", type=int, default=None, help="sequence length (default per workload)")
    ap.add_argument("--blocks", type=int, default=None, help="blocks for dit_step (default 40)")
    ap.add_argument("--rows", type=int, default=None, help="rows M of the linear / quant / S of the fused workload")
    ap.add_argument("--cols", type=int, default=None, help="columns K of the quant workload")
    ap.add_argument("--act", choices=["none", "gelu"], default="none", help="quant workload: activation")
    ap.add_argument("--exchange", choices=["p2p", "nccl"], default=os.environ.get("H3B_EXCHANGE", "p2p"))
    ap.add_argument("--overlap", type=int, default=None,
                    help="head groups of the exchange/attention overlap (default: H3B_SP_OVERLAP_GROUPS or the "
                         "reference's MINIMAX_SP_OVERLAP_CHUNKS; 0 = off)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-parity", action="store_true", help="skip the checker leg after the timed regions")
    ap.add_argument("--no-step", action="store_true", help="dit_block: skip the 40-block step sub-record")
    ap.add_argument("--no-a2a", action="store_true", help="dit_block at N > 1: skip the a2a sub-record")
    return ap.parse_args()


def peaks():
    try:
        with open(PEAKS_FILE) as f:
            p = json.load(f)
        return p, "measured"
    except (OSError, ValueError):
        return FALLBACK_PEAKS, "fallback"


# ---------------------------------------------------------------------------
# clocks sampled during the timed region

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.proc = None
        self.sel = []
        try:
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            self.sel = ["-i", uuid if uuid.startswith("GPU-") else "GPU-" + uuid]
        except Exception:  # noqa: BLE001
            self.sel = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", *self.sel, f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.rows = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=10)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            for line in out.splitlines():
                parts = [p.strip() for p in line.split(",")]
                if len(parts) == 9:
                    self.rows.append(parts)
        return False

    def summary(self):
        rows = getattr(self, "rows", [])
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["clock sampling unavailable"], "samples": 0}

        def num(v):
            try:
                return float(v)
            except ValueError:
                return None
        sm = [num(r[1]) for r in rows if num(r[1]) is not None]
        smax = [num(r[2]) for r in rows if num(r[2]) is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": reasons, "samples": len(rows),
                "power_w_max": max((num(r[3]) or 0.0) for r in rows)}


# ---------------------------------------------------------------------------
# distributed setup

def setup_dist(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        if world == 1 and args.gpus > 1:
            raise SystemExit("for --gpus N > 1 launch with torch.distributed.run (one process per GPU)")
    return rank, world, local


def init_pg(rank, world, local):
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=180),
                                device_id=dev)
    return dev


def max_over_ranks(v, world, dev):
    if world == 1:
        return v
    t = torch.tensor([v], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def timed(step, steps, warmup, world, dev, sample_clocks=True, finish=None):
    for _ in range(warmup):
        step()
    if finish is not None:
        finish()
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier(device_ids=[dev.index])
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(dev) if sample_clocks else None
    if sampler:
        sampler.__enter__()
        time.sleep(0.3)
    e0.record()
    for _ in range(steps):
        step()
    if finish is not None:
        finish()  # e.g. join side streams, so e1 follows all of the steps' work
    e1.record()
    torch.cuda.synchronize(dev)
    if sampler:
        sampler.__exit__(None, None, None)
    if world > 1:
        dist.barrier(device_ids=[dev.index])
    ms = e0.elapsed_time(e1) / steps
    return max_over_ranks(ms, world, dev), (sampler.summary() if sampler else None)


# ---------------------------------------------------------------------------
# synthetic inputs (seeded on CPU in row chunks, so every world size sees the same rows)

ROW_CHUNK = 4128  # one latent frame of tokens


def seeded_rows(start, stop, dim, seed, dtype=torch.bfloat16):
    out = torch.empty(stop - start, dim, dtype=dtype)
    c0 = start // ROW_CHUNK
    for c in range(c0, (stop + ROW_CHUNK - 1) // ROW_CHUNK):
        lo, hi = c * ROW_CHUNK, (c + 1) * ROW_CHUNK
        g = torch.Generator().manual_seed(seed * 7919 + c)
        block = torch.randn(ROW_CHUNK, dim, generator=g).to(dtype)
        a, b = max(lo, start), min(hi, stop)
        out[a - start:b - start] = block[a - lo:b - lo]
    return out


# ---------------------------------------------------------------------------
# DiT block / step workload

def gemm_shapes(cfg, s_local, world, exchange):
    """(M, N, K) of the launches the "gemm" span covers in one block: out, up and
    down always; qkv too unless it runs as the fused GEMM + exchange (its own span)."""
    from h3b import model as hm
    shapes = [(s_local, cfg.dim, cfg.dim), (s_local, cfg.ffn, cfg.dim), (s_local, cfg.dim, cfg.ffn)]
    fused_qkv = world > 1 and exchange == "p2p" and hm.FUSED_EXCHANGE and overlap_groups(cfg, world) == 0
    return shapes if fused_qkv else [(s_local, 3 * cfg.dim, cfg.dim)] + shapes


def overlap_groups(cfg, world):
    """Head groups the block's attention uses (0: exchange and attention in sequence).
    Reads the same environment as h3b.sp.overlap_groups without loading the
    library (the reference arm reports the same config)."""
    if world == 1:
        return 0
    hp = cfg.heads // world

    def env(name):
        return int(os.environ.get(name, "0") or 0)
    n = env("H3B_SP_OVERLAP_GROUPS") or env("MINIMAX_SP_OVERLAP_CHUNKS")
    if world == 4:
        n = env("MINIMAX_SP_OVERLAP_CHUNKS_W4") or n
        while n > 1 and hp % n:
            n -= 1
    return n if n > 1 and hp % n == 0 else 0


def dit_config(cfg, workload, seq, world, n_blocks, text_len, exchange):
    """The `config` object of a DiT line (both arms print the same one)."""
    base, rem = divmod(seq, world)
    return {"workload": workload, "seq_len": seq, "local_rows": base + (1 if rem else 0), "dim": cfg.dim,
            "heads": cfg.heads, "head_dim": cfg.head_dim, "ffn": cfg.ffn, "blocks": n_blocks, "text_len": text_len,
            "parallelism": f"ulysses_sp{world}", "exchange": exchange if world > 1 else None,
            "overlap_groups": overlap_groups(cfg, world), "l2": "inputs larger than L2 (no flush)"}


def dit_workload(args, rank, world, dev, n_blocks, seq, text_len, steps, warmup, trace=True, e2e_steps=None,
                 serial=True, parity=True, warm_blocks=0):
    """Times `steps` forwards of an n_blocks synthetic DiT over seq tokens
    (this rank's rows).  warmup full steps (or, with warm_blocks, that many
    single-block forwards, which run every kernel and shape of a step) come
    first.  Returns a dict: cfg, s_local, ms, clocks, spans/launches (trace),
    e2e (HostPipeline, e2e_steps steps; None skips it) and parity (the
    checker leg after all timed regions)."""
    import h3b
    from h3b import model as hm
    from h3b.trace import Trace

    if args.overlap is not None:
        os.environ["H3B_SP_OVERLAP_GROUPS"] = str(args.overlap)
    cfg = hm.DiTConfig(n_blocks=n_blocks, text_len=text_len)
    dit = hm.SynthDiT(cfg, dev, seed=1)
    peer = None
    ctx = None
    if world > 1:
        if args.exchange == "p2p":
            peer = h3b.PeerExchange(dist.group.WORLD, rank, world, seq, cfg.heads, cfg.head_dim)
        ctx = h3b.SPContext(rank, world, dist.group.WORLD, seq, exchange=args.exchange, peer=peer)
        h3b.startup_probe(rank, world, dist.group.WORLD, dev, peer=peer)
        start, stop = ctx.start, ctx.stop
    else:
        start, stop = 0, seq
    s_local = stop - start
    x_host = seeded_rows(start, stop, cfg.dim, seed=11).pin_memory()
    text_host = seeded_rows(0, text_len, cfg.dim, seed=12).pin_memory() if text_len else None
    x0 = x_host.to(dev)
    text = text_host.to(dev) if text_len else None
    xw = torch.empty_like(x0)
    ridx = torch.zeros(s_local, dtype=torch.int32, device=dev)
    res = {"cfg": cfg, "s_local": s_local, "spans": {}, "launches": 0, "e2e": None, "parity": None}

    def step():
        xw.copy_(x0)
        dit.forward(xw, ridx, ctx, text)

    for _ in range(warm_blocks):
        xw.copy_(x0)
        hm.block_forward(cfg, dit.params[0], xw, ridx, ctx, text)
    res["ms"], res["clocks"] = timed(step, steps, warmup, world, dev)
    if trace:
        # per-kernel spans over a second, identical timed region (events inside it)
        with Trace() as tr:
            timed(step, steps, 0, world, dev, sample_clocks=False)
        res["spans"], res["launches"] = tr.summary(steps), tr.launches / steps

    if e2e_steps:
        e_host = [p.e.detach().cpu().pin_memory() for p in dit.params]

        def load_tables(cond=None):
            # the step's adaLN conditioning: from its device copies (pipelined) or from the host (serial)
            for p, e in zip(dit.params, cond if cond is not None else e_host):
                p.e.copy_(e, non_blocking=True)
                p.tables = h3b.modulation_tables(*(p.e[:, i] for i in range(6)))

        # pipelined: HostPipeline, input copy (latent rows and conditioning) of step k+1 / output copy
        # of step k-1 on copy streams during step k (three device slots)
        pipe = hm.HostPipeline(dit, s_local, ridx, ctx, text, depth=3, timing=True)
        outs = [torch.empty_like(x_host).pin_memory() for _ in range(3)]

        def step_pipe():
            pipe.submit(x_host, outs[pipe.k % 3], before=load_tables, cond_host=e_host)

        ms_e2e, _ = timed(step_pipe, e2e_steps, 1 if serial else 0, world, dev, sample_clocks=False,
                          finish=pipe.flush)
        ct = pipe.copy_times()
        del pipe
        out_host = outs[0]
        h2d = x_host.numel() * 2 + sum(e.numel() * 2 for e in e_host)
        e2e = {"value": round(ms_e2e, 3), "unit": "ms/step", "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": out_host.numel() * 2,
               "api": "h3b.model.HostPipeline.submit (pinned host latents in and out; copies on two copy streams "
                      "overlap the neighbouring steps' compute, every step's copies inside the timed region)"}
        if ct["in"] and ct["out"]:
            # each rank's own copies (CUDA events on the copy streams), warm-up step included
            e2e["copy_in_ms"], e2e["copy_out_ms"] = round(ct["in"], 3), round(ct["out"], 3)
            e2e["copy_in_gbs"] = round(x_host.numel() * 2 / ct["in"] / 1e6, 1)
            e2e["copy_out_gbs"] = round(x_host.numel() * 2 / ct["out"] / 1e6, 1)
        if serial:
            # serial: copy in, forward, copy out, all on the compute stream
            def step_serial():
                load_tables()
                xw.copy_(x_host, non_blocking=True)
                y = dit.forward(xw, ridx, ctx, text)
                out_host.copy_(y, non_blocking=True)

            ms_serial, _ = timed(step_serial, e2e_steps, 1, world, dev, sample_clocks=False)
            e2e["serial_ms_per_step"] = round(ms_serial, 3)
        res["e2e"] = e2e
        del outs, out_host
    status = h3b.status()
    if status:
        raise RuntimeError(f"device status {status} after the timed region")
    if parity:
        # xw holds the output of the last forward of x0's rows (a timed step or a serial e2e step)
        res["parity"] = dit_parity(dit, x0, xw, ridx, text, rank, world, dev, seq, ctx)
    if peer is not None:
        torch.cuda.synchronize(dev)
        dist.barrier(device_ids=[dev.index])
        peer.close()
    del dit, x0, xw
    torch.cuda.empty_cache()
    return res


def dit_parity(dit, x0, y, ridx, text, rank, world, dev, seq, ctx):
    """Checker leg, run after every timed region: y, the timed path's output for
    the step's input rows x0, against the reference's eager PyTorch path
    (oracle/torch_path.py, which restates the eager DiTBlock sequence of
    h3_fuse_kernels.py:3-7, the INT8 linear of int8_gemm_triton.py:2,61-66 with
    torch._int_mm, SDPA, and at N > 1 the exchange of sp_forward.py:158-198 as
    reshape + all_to_all_single over NCCL), same weights and rows, every block
    of the model, compared bit for bit on every rank (mismatches summed over
    ranks)."""
    import h3b
    from oracle import torch_path as tp

    ctx_ref = h3b.SPContext(rank, world, dist.group.WORLD, seq) if world > 1 else None  # NCCL all_to_all_single
    xe = x0.clone()
    for p in dit.params:
        xe = tp.block_forward(dit.cfg, p, xe, ridx, ctx_ref, text)
    torch.cuda.synchronize(dev)
    bad = (y.view(torch.int16) != xe.view(torch.int16)).sum().to(torch.float64)
    nonfinite = (~torch.isfinite(y.float())).sum().to(torch.float64)
    counts = torch.stack([bad, nonfinite])
    if world > 1:
        dist.all_reduce(counts)
    mismatches, nonfinite = int(counts[0].item()), int(counts[1].item())
    del xe
    torch.cuda.empty_cache()
    return {"block_bitexact": mismatches == 0, "mismatches": mismatches, "elements": seq * dit.cfg.dim,
            "nonfinite": nonfinite, "blocks": len(dit.params),
            "exchange": None if world == 1 else getattr(ctx, "exchange", "nccl"),
            "reference": "eager PyTorch block (F.rms_norm/mul/add chain, torch._int_mm INT8 linears, SDPA"
                         + (", reshape + all_to_all_single over NCCL)" if world > 1 else ")")
                         + " on the same weights and rows, after the timed regions"}


def gemm_dram_traffic(shapes):
    """DRAM bytes per GEMM launch, averaged over the step's launches: each shape's
    algorithmic bytes (A + B + bf16 out + scales + bias) times the DRAM/algorithmic
    ratio that profiles/ncu_traffic.json records for its (N, K) from an ncu capture
    of a smaller M (the operand, re-read and output bytes all grow in proportion
    to M); shapes without a recorded ratio use the "default" entry."""
    try:
        with open(os.path.join(ROOT, "profiles", "ncu_traffic.json")) as f:
            rec = json.load(f)
    except (OSError, ValueError):
        return None, None
    ratios = {tuple(e["nk"]): e["ratio"] for e in rec.get("shapes", [])}
    default = rec.get("default", {}).get("ratio")
    total, used = 0.0, []
    for M, N, K in shapes:
        r = ratios.get((N, K), default)
        if r is None:
            return None, None
        used.append(round(r, 3))
        total += r * (M * K + N * K + 2 * M * N + 4 * M + 6 * N)
    return total / len(shapes), used


def gemm_roofline(spans, pk, src, shapes=None, in_step=False):
    """Roofline of the INT8 GEMM launches of the timed region.  Peak: 2 x the
    measured dense bf16 rate (kind::i8 issues at twice kind::f16), the sustained
    figure for launches timed inside a long step (power-capped clocks), the burst
    figure for a GEMM timed alone."""
    g = spans.get("gemm")
    if not g or g["ms"] <= 0:
        return None
    achieved = g["work"] / (g["ms"] * 1e-3) / 1e12  # TOPS
    key = "bf16_tflops_sustained" if in_step else "bf16_tflops"
    peak = 2.0 * pk[key]
    traffic, ratios = gemm_dram_traffic(shapes) if shapes else (None, None)
    return {"kernel": "gemm_i8_pair_kernel (tcgen05 cta_group::2 kind::i8 + dequant epilogue)", "bound": "tensor",
            "achieved": round(achieved, 1), "peak": round(peak, 1), "unit": "TOPS",
            "frac": round(achieved / peak, 4), "traffic": None if traffic is None else int(traffic),
            "traffic_note": None if ratios is None else
            f"bytes per launch (mean over the step's shapes): algorithmic operand+output bytes x the DRAM/algorithmic "
            f"ratio per (N, K) from profiles/ncu_traffic.json ({ratios})",
            "peak_source": f"2 x {src} bf16 dense, {'sustained' if in_step else 'burst'} ({pk[key]} TFLOP/s; "
                           "kind::i8 issues at twice the kind::f16 rate on B200)",
            "work_per_step": g["work"], "launches_per_step": g["calls"], "ms_per_step": round(g["ms"], 3)}


def int8_library_rate(dev, sustained_s=1.5):
    """The INT8 tensor rate of the box's own library GEMM, measured here:
    torch._int_mm (cuBLASLt, int8 x int8 -> int32, no epilogue) at 8192^3 --
    "burst": the best of 10 launches timed alone; "sustained": back to back for
    about sustained_s seconds (power-capped clocks, like a GEMM inside the
    step).  A reference beside the 2 x bf16 figure, which is inferred."""
    n = 8192
    g = torch.Generator(device=dev).manual_seed(2)
    a = torch.randint(-127, 128, (n, n), generator=g, dtype=torch.int8, device=dev)
    b = torch.randint(-127, 128, (n, n), generator=g, dtype=torch.int8, device=dev)
    ops = 2.0 * n ** 3
    for _ in range(3):
        torch._int_mm(a, b.t())
    best = None
    for _ in range(10):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        torch._int_mm(a, b.t())
        e1.record()
        torch.cuda.synchronize(dev)
        ms = e0.elapsed_time(e1)
        best = ms if best is None else min(best, ms)
    reps = max(1, int(sustained_s * 1e3 / best))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        torch._int_mm(a, b.t())
    e1.record()
    torch.cuda.synchronize(dev)
    sus = e0.elapsed_time(e1) / reps
    del a, b
    torch.cuda.empty_cache()
    return {"gemm": "torch._int_mm (cuBLASLt) 8192^3 int8 -> int32", "burst_tops": round(ops / best / 1e9, 1),
            "sustained_tops": round(ops / sus / 1e9, 1), "sustained_launches": reps}


def breakdown(spans, pk):
    out = {}
    for name, d in sorted(spans.items()):
        item = {"ms_per_step": round(d["ms"], 3), "calls_per_step": d["calls"]}
        if d["ms"] > 0 and d["work"] > 0:
            if name.startswith("gemm"):
                item["achieved_tops"] = round(d["work"] / (d["ms"] * 1e-3) / 1e12, 1)
            elif name == "sdpa":  # PyTorch's attention kernel (not this library's), bf16 tensor flops
                tf = d["work"] / (d["ms"] * 1e-3) / 1e12
                item["achieved_tflops"] = round(tf, 1)
                item["bf16_sustained_frac"] = round(tf / pk["bf16_tflops_sustained"], 3)
            elif name.startswith("a2a_fwd_p2p") or name.startswith("a2a_inv_p2p"):
                item["off_rank_gbs"] = round(d["work"] / (d["ms"] * 1e-3) / 1e9, 1)
            else:
                gbs = d["work"] / (d["ms"] * 1e-3) / 1e9
                item["achieved_gbs"] = round(gbs, 1)
                item["hbm_frac"] = round(gbs / pk["hbm_gbs"], 3)
        out[name] = item
    return out


# ---------------------------------------------------------------------------
# CPU reference path (eager PyTorch on the host cores), bounded sample

class CpuReference:
    """The reference's eager PyTorch path on the host cores, on a bounded sample.

    Row-local work (norms, INT8 linears, GELU, gates) is timed on rows_lo and
    rows_hi rows and attention on q_lo and q_hi query rows against all `seq`
    keys/values of every head; each part is extrapolated to the full sequence by
    the straight line through its two points (a fixed cost -- the layout copies
    of K and V inside SDPA, thread start-up -- plus a cost per row), so the
    fixed costs are counted once, not once per sampled fraction.  Set-up
    (weights, inputs) happens once; run() times one sample and returns the
    extrapolated ms per step."""

    def __init__(self, cfg, seq, rows=(1024, 4096), q_rows=(2048, 8192)):
        from types import SimpleNamespace as NS

        from oracle import torch_path as tp

        torch.set_num_threads(os.cpu_count() or 1)
        self.cfg, self.seq = cfg, seq
        self.rows, self.q_rows = tuple(min(r, seq) for r in rows), tuple(min(q, seq) for q in q_rows)
        g = torch.Generator().manual_seed(5)
        D, H, Dh = cfg.dim, cfg.heads, cfg.head_dim

        def lin(n, k):  # random-init INT8 linear of the benchmark block (same distributions as the GPU arm)
            return NS(w=torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8),
                      ws=(torch.rand(n, generator=g) + 0.5) / (127.0 * k ** 0.5),
                      b=(torch.randn(n, generator=g) * 0.02).to(torch.bfloat16))

        e = (0.1 * torch.randn(1, 6, D, generator=g)).to(torch.bfloat16)
        self.p = NS(n1w=(1 + 0.02 * torch.randn(D, generator=g)).to(torch.bfloat16),
                    n2w=(1 + 0.02 * torch.randn(D, generator=g)).to(torch.bfloat16),
                    qkv=lin(3 * D, D), out=lin(D, D), up=lin(cfg.ffn, D), down=lin(D, cfg.ffn),
                    tables=tp.modulation_tables(*(e[:, i] for i in range(6))))
        self.x = torch.randn(max(self.rows), D, generator=g).to(torch.bfloat16)
        self.ridx = torch.zeros(max(self.rows), dtype=torch.int32)
        self.q = torch.randn(max(self.q_rows), H, Dh, generator=g).to(torch.bfloat16)
        self.k = torch.randn(seq, H, Dh, generator=g).to(torch.bfloat16)
        self.v = torch.randn(seq, H, Dh, generator=g).to(torch.bfloat16)

    def _rowwork(self, n):
        import torch.nn.functional as F

        from oracle import torch_path as tp
        p, cfg, D = self.p, self.cfg, self.cfg.dim
        s1a, sha, ga, s1m, shm, gm = p.tables
        xx, ridx = self.x[:n].clone(), self.ridx[:n]
        h = tp.norm_mod(xx, p.n1w, cfg.eps, ridx, s1a, sha)
        qkv = tp.linear(h, p.qkv.w, p.qkv.ws, p.qkv.b)
        o = tp.linear(qkv[:, :D], p.out.w, p.out.ws, p.out.b)  # out-proj on an attention-output-sized input
        h = tp.gate_norm_mod_(xx, o, ga, p.n2w, cfg.eps, ridx, s1m, shm)
        u = tp.linear(h, p.up.w, p.up.ws, p.up.b)
        m = tp.linear(F.gelu(u, approximate="tanh"), p.down.w, p.down.ws, p.down.b)
        tp.gate_(xx, m, gm, ridx)

    def _attn(self, n):
        from oracle import torch_path as tp
        tp.sdpa_heads(self.q[:n], self.k, self.v)

    @staticmethod
    def _timed(fn, n):
        t0 = time.perf_counter()
        fn(n)
        return time.perf_counter() - t0

    def _line(self, fn, lo, hi):
        """Seconds for the full sequence from the line through (lo, t_lo) and (hi, t_hi)."""
        t_lo, t_hi = self._timed(fn, lo), self._timed(fn, hi)
        self.last_cpu_s += t_lo + t_hi
        if hi <= lo:
            return t_hi * self.seq / hi
        per_row = (t_hi - t_lo) / (hi - lo)
        if per_row <= 0.0:  # timing noise swamped the slope: plain proportional scaling (an upper bound)
            return t_hi * self.seq / hi
        return max(t_hi - per_row * hi, 0.0) + per_row * self.seq

    def run(self):
        self.last_cpu_s = 0.0
        rows_s = self._line(self._rowwork, *self.rows)
        attn_s = self._line(self._attn, *self.q_rows)
        return (rows_s + attn_s) * 1e3

    def sample(self):
        return (f"eager PyTorch CPU path (oracle/torch_path.py): row-local block work (norms, 4 INT8 linears, "
                f"GELU, gates) on {self.rows[0]} and {self.rows[1]} of {self.seq} rows, SDPA for {self.q_rows[0]} "
                f"and {self.q_rows[1]} query rows vs all {self.seq} keys, {self.cfg.heads} heads; each part "
                f"extrapolated to {self.seq} rows along the line through its two timings (fixed cost counted "
                f"once); {self.last_cpu_s:.1f} s of CPU work per sample")


def cpu_baseline(cfg, seq, steps=3, warmup=1):
    ref = CpuReference(cfg, seq)
    for _ in range(warmup):
        ref.run()
    runs = [ref.run() for _ in range(steps)]
    ms = statistics.median(runs)
    return {"value": round(ms, 1), "unit": "ms/step", "cores": torch.get_num_threads(), "kind": "port",
            "sample": ref.sample(), "runs_ms": [round(r, 1) for r in runs],
            "spread": round((max(runs) - min(runs)) / ms, 3)}


# ---------------------------------------------------------------------------
# by-hand workloads (configs 0-2)

def linear_workload(args, dev):
    import h3b
    from h3b.trace import Trace
    M, N, K = args.rows or 4096, 5120, 5120
    g = torch.Generator().manual_seed(0)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16).to(dev)
    w = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int8).to(dev)
    ws = (torch.rand(N, generator=g) * 9e-3 + 1e-3).to(dev)
    b = (torch.randn(N, generator=g) * 0.02).to(torch.bfloat16).to(dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def step():
        flush.zero_()
        h3b.linear(x, w, ws, b, convrot_group=args.convrot)

    ms, clocks = timed(step, args.steps, args.warmup, 1, dev)
    with Trace() as tr:
        timed(step, args.steps, 0, 1, dev, sample_clocks=False)
    return ms, clocks, tr.summary(args.steps), tr.launches / args.steps


def quant_workload(args, dev):
    """The activation quantiser alone (h3b_quant_rowwise, or with --act gelu the
    GELU-tanh quantiser h3b_gelu_quant that feeds the down projection) on
    seeded N(0,1) bf16 rows [M, K] (M*K*2 bytes > L2 at the default sizes)."""
    import h3b
    from h3b.trace import Trace
    M, K = args.rows or 32768, args.cols or (13824 if args.act == "gelu" else 5120)
    x = seeded_rows(0, M, K, seed=30).to(dev)
    xq = torch.empty(M, K, dtype=torch.int8, device=dev)
    xs = torch.empty(M, 1, dtype=torch.float32, device=dev)
    fn = h3b.gelu_quant if args.act == "gelu" else h3b.quant_rowwise

    def step():
        fn(x, xq, xs)

    ms, clocks = timed(step, args.steps, args.warmup, 1, dev)
    with Trace() as tr:
        timed(step, args.steps, 0, 1, dev, sample_clocks=False)
    return M, K, ms, clocks, tr.summary(args.steps), tr.launches / args.steps


def gemm_workload(args, dev):
    """The block's four INT8 GEMM shapes alone (qkv 5120->15360, out 5120->5120,
    up 5120->13824, down 13824->5120) at M rows (default 128000, the benchmark
    block), with bias, each launch timed with CUDA events after a 256 MB L2
    flush; returns [(name, M, N, K, ms)].  Inputs are drawn on the device
    (timing only)."""
    import h3b
    M = args.rows or 128000
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    out = []
    for name, N, K in (("qkv", 15360, 5120), ("out", 5120, 5120), ("up", 13824, 5120), ("down", 5120, 13824)):
        g = torch.Generator(device=dev).manual_seed(N + K)
        xq = torch.randint(-127, 128, (M, K), generator=g, dtype=torch.int8, device=dev)
        xs = torch.rand(M, 1, generator=g, device=dev) * 0.05 + 1e-3
        w = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int8, device=dev)
        ws = torch.rand(N, generator=g, device=dev) * 9e-3 + 1e-3
        b = (torch.randn(N, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        y = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
        ms = _event_time(lambda: h3b.int8_mm_scaled(xq, w, xs, ws, out=y, bias=b), args.steps, flush,
                         warmup=args.warmup)
        out.append((name, M, N, K, ms))
        del xq, xs, w, ws, b, y
        torch.cuda.empty_cache()
    return out


def qkv_a2a_workload(args, dev):
    """One rank's qkv projection with the forward exchange in the GEMM's epilogue
    (h3b_int8_mm_scaled_a2a), on one GPU: the P ranks' receive buffers are all
    local here, so this times the kernel with the scatter epilogue against the
    plain GEMM of the same shape (the NVLink leg is measured by the dit_block
    workload at N > 1)."""
    import h3b
    from h3b.trace import Trace
    P = args.peers
    M, D, H, Dh = args.rows or 16000, 5120, 40, 128
    hp = H // P
    g = torch.Generator().manual_seed(0)
    xq = torch.randint(-127, 128, (M, D), generator=g, dtype=torch.int8).to(dev)
    xs = (torch.rand(M, 1, generator=g) * 0.05 + 1e-3).to(dev)
    w = torch.randint(-127, 128, (3 * D, D), generator=g, dtype=torch.int8).to(dev)
    ws = (torch.rand(3 * D, generator=g) * 9e-3 + 1e-3).to(dev)
    b = (torch.randn(3 * D, generator=g) * 0.02).to(torch.bfloat16).to(dev)
    recv = [torch.empty(M, hp * Dh, dtype=torch.bfloat16, device=dev) for _ in range(3 * P)]  # rank 0's rows
    dst = [t.data_ptr() for t in recv]
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    nw = (1 + 0.02 * torch.randn(2, Dh, generator=g)).to(torch.bfloat16).to(dev) if args.qknorm else None

    def step():
        flush.zero_()
        h3b.int8_mm_scaled_a2a(xq, w, xs, ws, b, dst, 0, D, Dh, hp, P, norm_w=nw)

    def step_plain():
        flush.zero_()
        h3b.int8_mm_scaled(xq, w, xs, ws, bias=b)

    ms, clocks = timed(step, args.steps, args.warmup, 1, dev)
    for _ in range(args.warmup):
        step_plain()
    with Trace() as tr:
        timed(step, args.steps, 0, 1, dev, sample_clocks=False)
        timed(step_plain, args.steps, 0, 1, dev, sample_clocks=False)
    return M, ms, clocks, tr.summary(args.steps), tr.launches / args.steps


def fused_workload(args, dev):
    import h3b
    from h3b.trace import Trace
    S, D = args.rows or 32768, 5120
    x0 = seeded_rows(0, S, D, seed=3).to(dev)
    o1 = seeded_rows(0, S, D, seed=4).to(dev)
    o2 = seeded_rows(0, S, D, seed=5).to(dev)
    g = torch.Generator().manual_seed(6)
    e = (0.1 * torch.randn(1, 6, D, generator=g)).to(torch.bfloat16).to(dev)
    w1 = (1 + 0.02 * torch.randn(D, generator=g)).to(torch.bfloat16).to(dev)
    w2 = (1 + 0.02 * torch.randn(D, generator=g)).to(torch.bfloat16).to(dev)
    s1a, sha, ga, s1m, shm, gm = h3b.modulation_tables(*(e[:, i] for i in range(6)))
    ridx = torch.zeros(S, dtype=torch.int32, device=dev)
    x = torch.empty_like(x0)

    def step():
        x.copy_(x0)
        h3b.norm_mod(x, w1, 1e-6, ridx, s1a, sha)
        h3b.gate_norm_mod_(x, o1, ga, w2, 1e-6, ridx, s1m, shm)
        h3b.gate_(x, o2, gm, ridx)

    ms, clocks = timed(step, args.steps, args.warmup, 1, dev)
    with Trace() as tr:
        timed(step, args.steps, 0, 1, dev, sample_clocks=False)
    return ms, clocks, tr.summary(args.steps), tr.launches / args.steps


def a2a_workload(args, rank, world, dev):
    import h3b
    from h3b.trace import Trace
    S, H, Dh = args.seq or 131072, 40, 128
    peer = h3b.PeerExchange(dist.group.WORLD, rank, world, S, H, Dh) if args.exchange == "p2p" else None
    ctx = h3b.SPContext(rank, world, dist.group.WORLD, S, exchange=args.exchange, peer=peer)
    q, k, v = (seeded_rows(ctx.start, ctx.stop, H * Dh, seed=20 + i).to(dev).view(-1, H, Dh) for i in range(3))

    def step():
        qq, kk, vv = h3b.a2a_gather_qkv(q, k, v, ctx)
        h3b.a2a_scatter_seq_gather_heads(qq.reshape(S, -1), ctx)

    ms, clocks = timed(step, args.steps, args.warmup, world, dev)
    with Trace() as tr:
        timed(step, args.steps, 0, world, dev, sample_clocks=False)
    if peer is not None:
        torch.cuda.synchronize(dev)
        dist.barrier(device_ids=[dev.index])
        peer.close()
    return S, ms, clocks, tr.summary(args.steps), tr.launches / args.steps


def nvlink_probe_workload(args):
    """One process, two GPUs (no rank waits on another): rank 0's side of a
    2-rank forward exchange.  On GPU 0 the forward-exchange copy kernel
    (h3b_a2a_fwd_p2p, q/k/v [s_local, 40, 128]) and the qkv GEMM with the
    exchange in its epilogue (h3b_int8_mm_scaled_a2a) store half of their
    output into receive buffers on GPU 1 (peer access enabled) with plain
    stores, the other half locally; the host synchronises between launches.
    For ncu's NVLink byte counters next to CUDA-event timings; the payload that
    crosses NVLink is s_local x 3 x 2560 x 2 bytes per launch."""
    import ctypes

    import h3b
    from cuda.bindings import runtime as rt
    from h3b._lib import check, lib, ptr_array, stream_of
    if torch.cuda.device_count() < 2:
        raise SystemExit("the nvlink_probe workload needs 2 GPUs in one process")
    for a, b in ((0, 1), (1, 0)):
        torch.cuda.set_device(a)
        (err,) = rt.cudaSetDevice(a)
        (err,) = rt.cudaDeviceEnablePeerAccess(b, 0)
        if err not in (rt.cudaError_t.cudaSuccess, rt.cudaError_t.cudaErrorPeerAccessAlreadyEnabled):
            raise SystemExit(f"cudaDeviceEnablePeerAccess({a}->{b}) failed: {err}")
    d0, d1 = torch.device("cuda", 0), torch.device("cuda", 1)
    torch.cuda.set_device(d0)
    P, H, Dh = 2, 40, 128
    s_local = args.rows or 16384
    S, chunk = P * s_local, H // P * Dh
    src = [seeded_rows(0, s_local, H * Dh, seed=40 + i).to(d0) for i in range(3)]
    recv = [[torch.zeros(S, chunk, dtype=torch.bfloat16, device=d) for d in (d0, d1)] for _ in range(3)]
    dst = [recv[i][j].data_ptr() for i in range(3) for j in range(P)]
    off = s_local * chunk * 2 * 3  # bytes per launch that cross NVLink (the half for rank 1)
    src_arr, k1 = ptr_array([t.data_ptr() for t in src])
    dst_arr, k2 = ptr_array(dst)

    def copy():
        check(lib.h3b_a2a_fwd_p2p(3, src_arr, H * Dh * 2, dst_arr, s_local, 0, chunk * 2, chunk * 2, 0, P,
                                  stream_of(src[0])), "h3b_a2a_fwd_p2p")
    g = torch.Generator().manual_seed(0)
    xq = torch.randint(-127, 128, (s_local, H * Dh), generator=g, dtype=torch.int8).to(d0)
    xs = (torch.rand(s_local, 1, generator=g) * 0.05 + 1e-3).to(d0)
    w = torch.randint(-127, 128, (3 * H * Dh, H * Dh), generator=g, dtype=torch.int8).to(d0)
    ws = (torch.rand(3 * H * Dh, generator=g) * 9e-3 + 1e-3).to(d0)
    bias = (torch.randn(3 * H * Dh, generator=g) * 0.02).to(torch.bfloat16).to(d0)

    def gemm():
        h3b.int8_mm_scaled_a2a(xq, w, xs, ws, bias, dst, 0, H * Dh, Dh, H // P, P)
    res = {}
    ok = False
    for name, fn in (("a2a_fwd_p2p", copy), ("gemm_i8_scatter_qkv", gemm)):
        ms = _event_time(lambda: (fn(), torch.cuda.synchronize(d1)), args.steps, warmup=args.warmup)
        res[name] = {"ms": round(ms, 4), "nvlink_payload_bytes": off,
                     "nvlink_payload_gbs": round(off / ms / 1e6, 1)}
        if name == "a2a_fwd_p2p":  # before the GEMM overwrites the buffers: rank 1 holds heads 20..39 of rank 0's rows
            ok = all(torch.equal(recv[i][1][:s_local].view(torch.int16),
                                 src[i].view(s_local, P, chunk)[:, 1].contiguous().to(d1).view(torch.int16))
                     for i in range(3))
    del k1, k2
    return s_local, res, ok


def load_reference_triton():
    """The reference's own Triton kernel modules (int8_gemm_triton.py,
    h3_fuse_kernels.py), unmodified, from baseline/_ref/comfyui_nodes (the
    reference has no installable package for them; they are copied there as
    its install, git-ignored).  Returns {"gemm": module, "fuse": module} or
    None when they are absent (e.g. a checkout without the reference)."""
    import importlib.util
    base = os.path.join(ROOT, "baseline", "_ref", "comfyui_nodes")
    mods = {}
    for key, rel in (("gemm", os.path.join("h3-linear-fast", "int8_gemm_triton.py")),
                     ("fuse", os.path.join("h3-fuse-graph", "h3_fuse_kernels.py"))):
        path = os.path.join(base, rel)
        if not os.path.exists(path):
            return None
        spec = importlib.util.spec_from_file_location(f"h3ref_{key}", path)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        mods[key] = mod
    return mods


def _event_time(fn, iters, flush=None, warmup=3):
    """Mean ms of fn() over iters launches, each timed alone with CUDA events on
    the current stream (a flush of L2 before each, outside the events)."""
    for _ in range(warmup):
        fn()
    total = 0.0
    for _ in range(iters):
        if flush is not None:
            flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize()
        total += e0.elapsed_time(e1)
    return total / iters


def vs_triton_workload(args, dev, pk, pk_src):
    """Same-box comparison: the reference's Triton INT8 GEMM and fused norm
    kernels, this library's kernels and cuBLASLt (torch._int_mm + the eager
    epilogue) on identical seeded inputs on one B200, each launch timed alone
    with CUDA events after a 256 MB L2 flush; outputs compared bit for bit."""
    import h3b
    ref = load_reference_triton()
    if ref is None:
        return {"unavailable": "the reference's Triton modules are not under baseline/_ref/comfyui_nodes"}
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    it = args.steps
    out = {"gemm": [], "fused": [], "int_mm_peak": None}
    shapes = [("config0", 4096, 5120, 5120), ("m32768", 32768, 5120, 5120),
              ("block_qkv", 128000, 15360, 5120), ("block_out", 128000, 5120, 5120),
              ("block_up", 128000, 13824, 5120), ("block_down", 128000, 5120, 13824)]
    for name, M, N, K in shapes:
        g = torch.Generator().manual_seed(M + N + K)
        xq = torch.randint(-127, 128, (M, K), generator=g, dtype=torch.int8).to(dev)
        w = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int8).to(dev)
        xs = (torch.rand(M, 1, generator=g) * 0.05 + 1e-3).to(dev)
        ws = (torch.rand(N, generator=g) * 9e-3 + 1e-3).to(dev)
        y_ref = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
        y_ours = torch.empty_like(y_ref)
        t_ref = _event_time(lambda: ref["gemm"].int8_mm_scaled(xq, w, xs, ws, out=y_ref), it, flush)
        t_ours = _event_time(lambda: h3b.int8_mm_scaled(xq, w, xs, ws, out=y_ours), it, flush)

        def cublas():
            return ((torch._int_mm(xq, w.t()).float() * xs) * ws).to(torch.bfloat16)
        t_cub = _event_time(cublas, max(2, it // 2), flush, warmup=1)
        t_cub_mm = _event_time(lambda: torch._int_mm(xq, w.t()), it, flush)
        y_cub = cublas()
        torch.cuda.synchronize()
        ops = 2.0 * M * N * K
        rec = {"shape": name, "M": M, "N": N, "K": K,
               "ms": {"reference_triton": round(t_ref, 4), "h3b": round(t_ours, 4),
                      "cublaslt_int_mm_plus_eager_epilogue": round(t_cub, 4), "cublaslt_int_mm_only": round(t_cub_mm, 4)},
               "tops": {"reference_triton": round(ops / t_ref / 1e9, 1), "h3b": round(ops / t_ours / 1e9, 1),
                        "cublaslt_int_mm_only": round(ops / t_cub_mm / 1e9, 1)},
               "speedup_vs_reference_triton": round(t_ref / t_ours, 3),
               "speedup_vs_cublaslt_path": round(t_cub / t_ours, 3),
               "bitexact_vs_reference_triton": bool(torch.equal(y_ref.view(torch.int16), y_ours.view(torch.int16))),
               "bitexact_vs_cublaslt_path": bool(torch.equal(y_cub.view(torch.int16), y_ours.view(torch.int16)))}
        out["gemm"].append(rec)
        log(json.dumps(rec))
        del xq, w, xs, ws, y_ref, y_ours, y_cub
        torch.cuda.empty_cache()
    # a measured INT8 rate of the box's own library GEMM (cuBLASLt int8 -> int32), beside the 2 x bf16 peak
    n = 8192
    g = torch.Generator().manual_seed(1)
    a = torch.randint(-127, 128, (n, n), generator=g, dtype=torch.int8).to(dev)
    b = torch.randint(-127, 128, (n, n), generator=g, dtype=torch.int8).to(dev)
    t = _event_time(lambda: torch._int_mm(a, b.t()), it)
    out["int_mm_peak"] = {"shape": f"{n}^3 int8 -> int32 (torch._int_mm, cuBLASLt)", "tops": round(2.0 * n ** 3 / t / 1e9, 1),
                          "ms": round(t, 4), "vs_2x_bf16_burst": round(2.0 * n ** 3 / t / 1e9 / (2 * pk["bf16_tflops"]), 3)}
    del a, b
    # fused adaLN chain at configuration 1 (S=32768, D=5120, one modulation row)
    S, D = args.rows or 32768, 5120
    g = torch.Generator().manual_seed(6)
    x0 = seeded_rows(0, S, D, seed=3).to(dev)
    o1 = seeded_rows(0, S, D, seed=4).to(dev)
    e = (0.1 * torch.randn(1, 6, D, generator=g)).to(torch.bfloat16).to(dev)
    wn = (1 + 0.02 * torch.randn(D, generator=g)).to(torch.bfloat16).to(dev)
    s1, sh, gt = h3b.modulation_tables(*(e[:, i] for i in range(6)))[:3]
    ridx = torch.zeros(S, dtype=torch.int32, device=dev)
    xa, xb = x0.clone(), x0.clone()
    cases = [("norm_mod", 4 * S * D, lambda: ref["fuse"].norm_mod(xa, wn, 1e-6, ridx, s1, sh),
              lambda: h3b.norm_mod(xb, wn, 1e-6, ridx, s1, sh)),
             ("gate_norm_mod_", 8 * S * D, lambda: ref["fuse"].gate_norm_mod_(xa, o1, gt, wn, 1e-6, ridx, s1, sh),
              lambda: h3b.gate_norm_mod_(xb, o1, gt, wn, 1e-6, ridx, s1, sh)),
             ("gate_", 6 * S * D, lambda: ref["fuse"].gate_(xa, o1, gt, ridx), lambda: h3b.gate_(xb, o1, gt, ridx))]
    for name, nbytes, f_ref, f_ours in cases:
        # bit-equality on one call from the same state, then timing (the in-place ops keep changing x alike)
        xa.copy_(x0)
        xb.copy_(x0)
        h_ref, h_ours = f_ref(), f_ours()
        torch.cuda.synchronize()
        same = bool(torch.equal(h_ref.view(torch.int16), h_ours.view(torch.int16))) and \
            bool(torch.equal(xa.view(torch.int16), xb.view(torch.int16)))
        t_ref = _event_time(f_ref, it, flush)
        t_ours = _event_time(f_ours, it, flush)
        rec = {"kernel": name, "S": S, "D": D, "ms": {"reference_triton": round(t_ref, 4), "h3b": round(t_ours, 4)},
               "hbm_frac_of_measured": {"reference_triton": round(nbytes / t_ref / 1e6 / pk["hbm_gbs"], 3),
                                        "h3b": round(nbytes / t_ours / 1e6 / pk["hbm_gbs"], 3)},
               "speedup_vs_reference_triton": round(t_ref / t_ours, 3), "bitexact_vs_reference_triton": same}
        out["fused"].append(rec)
        log(json.dumps(rec))
    return out


def nvlink_counters(dev):
    """Cumulative NVLink bytes of this GPU from NVML (read-only counters), summed
    over its links: {"tx": bytes, "rx": bytes, "field": name} or None.  Tries the
    per-link byte counters, then the per-link data throughput counters (KiB)."""
    try:
        import pynvml as nv
        nv.nvmlInit()
        uuid = str(torch.cuda.get_device_properties(dev).uuid)
        h = nv.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
        links = getattr(nv, "NVML_NVLINK_MAX_LINKS", 18)
        for name, tx_id, rx_id, scale in (
                ("NVML_FI_DEV_NVLINK_COUNT_XMIT_BYTES/RCV_BYTES", nv.NVML_FI_DEV_NVLINK_COUNT_XMIT_BYTES,
                 nv.NVML_FI_DEV_NVLINK_COUNT_RCV_BYTES, 1),
                ("NVML_FI_DEV_NVLINK_THROUGHPUT_DATA_TX/RX (KiB)", nv.NVML_FI_DEV_NVLINK_THROUGHPUT_DATA_TX,
                 nv.NVML_FI_DEV_NVLINK_THROUGHPUT_DATA_RX, 1024)):
            ids = [(tx_id, li) for li in range(links)] + [(rx_id, li) for li in range(links)]
            vals = nv.nvmlDeviceGetFieldValues(h, ids)
            ok = [v.nvmlReturn == 0 for v in vals]
            if not any(ok):
                continue
            tx = sum(int(v.value.ullVal) for v, o in zip(vals[:links], ok[:links]) if o) * scale
            rx = sum(int(v.value.ullVal) for v, o in zip(vals[links:], ok[links:]) if o) * scale
            return {"tx": tx, "rx": rx, "field": name, "links_read": sum(ok) // 2}
    except Exception as e:  # noqa: BLE001
        log(f"NVML NVLink counters unavailable: {e}")
    return None


def a2a_subrecord(args, rank, world, dev, seq=131072, steps=10, warmup=3):
    """Configuration 2 at this world size: q, k, v [S/P, 40, 128] forward
    exchange + inverse exchange of the received q (an identity round trip), per
    back end; bus GB/s = 4 tensors x the per-rank buffer x (P-1)/P / time (the
    all-to-all convention).  The round trip is checked bit for bit after the
    timed region; NVML's NVLink byte counters are read around it."""
    import h3b
    H, Dh = 40, 128
    out = {}
    for exch in ("p2p", "nccl"):
        peer = h3b.PeerExchange(dist.group.WORLD, rank, world, seq, H, Dh) if exch == "p2p" else None
        ctx = h3b.SPContext(rank, world, dist.group.WORLD, seq, exchange=exch, peer=peer)
        q, k, v = (seeded_rows(ctx.start, ctx.stop, H * Dh, seed=20 + i).to(dev).view(-1, H, Dh) for i in range(3))
        res = {}

        def step():
            qq, kk, vv = h3b.a2a_gather_qkv(q, k, v, ctx)
            res["back"] = h3b.a2a_scatter_seq_gather_heads(qq.reshape(seq, -1), ctx)

        for _ in range(warmup):
            step()
        torch.cuda.synchronize(dev)
        c0 = nvlink_counters(dev)
        ms, _ = timed(step, steps, 0, world, dev, sample_clocks=False)
        c1 = nvlink_counters(dev)
        buf = seq // world * H * Dh * 2
        bus = 4 * buf * (world - 1) / world / (ms * 1e-3) / 1e9
        step()
        torch.cuda.synchronize(dev)
        bad = (res["back"].reshape(-1).view(torch.int16) != q.reshape(-1).view(torch.int16)).sum().to(torch.float64)
        dist.all_reduce(bad)
        rec = {"bus_gbs": round(bus, 1), "ms_per_step": round(ms, 4), "steps": steps, "warmup": warmup,
               "link_peak_gbs": 900.0, "frac_of_900": round(bus / 900.0, 3),
               "roundtrip_bitexact": int(bad.item()) == 0, "roundtrip_mismatches": int(bad.item())}
        if c0 and c1:
            tx = (c1["tx"] - c0["tx"]) / steps
            rx = (c1["rx"] - c0["rx"]) / steps
            rec["nvml_nvlink"] = {"tx_bytes_per_step": tx, "rx_bytes_per_step": rx, "field": c0["field"],
                                  "links_read": c0["links_read"],
                                  "tx_gbs": round(tx / (ms * 1e-3) / 1e9, 1),
                                  "payload_off_rank_bytes_per_step": 4 * buf * (world - 1) / world}
        out[exch] = rec
        if peer is not None:
            torch.cuda.synchronize(dev)
            dist.barrier(device_ids=[dev.index])
            peer.close()
        del q, k, v, res
    torch.cuda.empty_cache()
    return {"metric": "Ulysses a2a bus GB/s (q,k,v forward + inverse)", "unit": "GB/s",
            "config": {"workload": "a2a", "S": seq, "heads": H, "head_dim": Dh, "world": world}, **out}


# ---------------------------------------------------------------------------

def main():
    args = parse_args()
    rank, world, local = setup_dist(args)
    pk, pk_src = peaks()

    if args.impl == "reference":
        if rank != 0:
            return
        from types import SimpleNamespace
        seq = args.seq or 128000
        # the benchmark block's shape (the reference arm loads nothing of this library)
        cfg = SimpleNamespace(dim=5120, heads=40, head_dim=128, ffn=13824, eps=1e-6)
        ref = CpuReference(cfg, seq)
        for _ in range(args.warmup):
            ref.run()
        runs = [ref.run() for _ in range(args.steps)]
        v = statistics.median(runs)
        sample, cores = ref.sample(), torch.get_num_threads()
        line = {"impl": "reference", "metric": "DiT fwd ms/step", "value": round(v, 1), "unit": "ms/step",
                "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(v, 1),
                "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "int8+bf16",
                "data": "synthetic (seeded N(0,1) activations, random-init int8 weights)",
                "config": dit_config(cfg, "dit_block", seq, args.gpus, 1, 0, args.exchange),
                "host": "CPU (the reference's eager PyTorch path on the host cores; rank 0 only)",
                "cpu_baseline": {"value": round(v, 1), "unit": "ms/step", "cores": cores, "kind": "port",
                                 "sample": sample, "spread": round((max(runs) - min(runs)) / v, 3),
                                 "runs_ms_min_max": [round(min(runs), 1), round(max(runs), 1)]},
                "e2e": {"value": round(v, 1), "unit": "ms/step", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    dev = init_pg(rank, world, local)
    try:
        if args.workload in ("dit_block", "dit_step"):
            step_cfg = args.workload == "dit_step"
            seq = args.seq or (252000 if step_cfg else 128000)
            n_blocks = args.blocks or (40 if step_cfg else 1)
            text_len = 512 if step_cfg else 0
            r = dit_workload(args, rank, world, dev, n_blocks, seq, text_len, args.steps, args.warmup,
                             e2e_steps=None if args.no_e2e else args.steps, parity=not args.no_parity)
            cfg, s_local, ms, spans = r["cfg"], r["s_local"], r["ms"], r["spans"]
            line = {"metric": "DiT fwd ms/step", "value": round(ms, 3), "unit": "ms/step", "n_gpus": world,
                    "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
                    "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "int8+bf16",
                    "data": "synthetic (seeded N(0,1) activations, random-init int8 weights)",
                    "config": dit_config(cfg, args.workload, seq, world, n_blocks, text_len, args.exchange),
                    "roofline": gemm_roofline(spans, pk, pk_src, gemm_shapes(cfg, s_local, world, args.exchange),
                                              in_step=True),
                    "clocks": r["clocks"], "e2e": r["e2e"], "parity": r["parity"],
                    "gpu_launches": int(round(r["launches"] * args.steps)), "breakdown": breakdown(spans, pk)}
            rl = line["roofline"]
            if rl is not None:
                # the GEMM against a measured INT8 rate of this GPU as well (cuBLASLt, timed after the timed regions)
                lib = int8_library_rate(dev)
                rl["int8_library_measured"] = lib
                rl["frac_of_library_sustained"] = round(rl["achieved"] / lib["sustained_tops"], 4)
            if rank == 0 and world == 1 and not args.no_cpu_baseline and not step_cfg:
                line["cpu_baseline"] = cpu_baseline(cfg, seq)
            if not step_cfg and world > 1 and not args.no_a2a:
                line["a2a"] = a2a_subrecord(args, rank, world, dev)
            if not step_cfg and not args.no_step:
                # configuration 4 (the 40-block step with 512 text tokens) as a sub-record: one block
                # forward warms every kernel and shape of the step, then 2 timed steps, 1 step end to end
                # through HostPipeline, and the final latent checked against the eager path
                rs = dit_workload(args, rank, world, dev, 40, 252000, 512, 2, 0, trace=False,
                                  e2e_steps=None if args.no_e2e else 1, serial=False,
                                  parity=not args.no_parity, warm_blocks=1)
                line["dit_step"] = {
                    "metric": "DiT fwd ms/step (40-block step)", "value": round(rs["ms"], 1), "unit": "ms/step",
                    "steps": 2, "warmup": "1 block forward (every kernel and shape of the step)",
                    "config": dit_config(rs["cfg"], "dit_step", 252000, world, 40, 512, args.exchange),
                    "clocks": rs["clocks"], "e2e": rs["e2e"], "parity": rs["parity"]}
        elif args.workload == "linear":
            ms, clocks, spans, launches = linear_workload(args, dev)
            M = args.rows or 4096
            rl = gemm_roofline(spans, pk, pk_src, [(M, 5120, 5120)])
            # the linear's own time: the quantiser and GEMM spans (the step also holds the L2 flush)
            lin_ms = sum(d["ms"] for k, d in spans.items() if k.startswith(("quant", "gemm")))
            line = {"metric": "INT8 linear (config 0) TOPS", "value": round(2 * M * 5120 * 5120 / (lin_ms * 1e-3) / 1e12, 1),
                    "unit": "TOPS", "ms_per_step": round(lin_ms, 4), "step_ms_with_flush": round(ms, 4),
                    "n_gpus": 1, "steps": args.steps,
                    "warmup": args.warmup, "higher_is_better": True, "dtype": "int8",
                    "config": {"workload": "linear", "M": M, "N": 5120, "K": 5120, "convrot_group": args.convrot,
                               "l2": "256 MB flush per step"},
                    "roofline": rl, "clocks": clocks, "gpu_launches": int(round(launches * args.steps)),
                    "breakdown": breakdown(spans, pk)}
        elif args.workload == "gemm":
            res = gemm_workload(args, dev)
            peak = 2.0 * pk["bf16_tflops"]
            shapes = [{"shape": n, "M": M, "N": N, "K": K, "ms": round(ms, 4),
                       "tops": round(2.0 * M * N * K / ms / 1e9, 1),
                       "frac_of_2x_bf16_burst": round(2.0 * M * N * K / ms / 1e9 / peak, 4)} for n, M, N, K, ms in res]
            tot_ms = sum(r[4] for r in res)
            tot_ops = sum(2.0 * r[1] * r[2] * r[3] for r in res)
            line = {"metric": "block INT8 GEMMs TOPS", "value": round(tot_ops / tot_ms / 1e9, 1), "unit": "TOPS",
                    "ms_per_step": round(tot_ms, 4), "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
                    "higher_is_better": True, "dtype": "int8",
                    "config": {"workload": "gemm", "M": res[0][1], "group_m": os.environ.get("H3B_GEMM_GROUP_M"),
                               "l2": "256 MB flush before each launch"},
                    "shapes": shapes}
        elif args.workload == "nvlink_probe":
            s_local, res, ok = nvlink_probe_workload(args)
            line = {"metric": "forward exchange over NVLink, one process driving 2 GPUs (GB/s of payload)",
                    "n_gpus": 2, "steps": args.steps, "warmup": args.warmup,
                    "config": {"workload": "nvlink_probe", "s_local": s_local, "heads": 40, "head_dim": 128,
                               "world": 2, "link_peak_gbs": 900.0},
                    "payload_bitexact": ok, **res}
        elif args.workload == "vs_triton":
            res = vs_triton_workload(args, dev, pk, pk_src)
            line = {"metric": "same-box comparison with the reference's Triton kernels", "n_gpus": 1,
                    "steps": args.steps, "config": {"workload": "vs_triton", "l2": "256 MB flush before each launch"},
                    "peak_source": f"{pk_src} (MEASURED_PEAKS.json: HBM {pk['hbm_gbs']} GB/s, bf16 {pk['bf16_tflops']} "
                                   "TFLOP/s burst)", **res}
        elif args.workload == "quant":
            M, K, ms, clocks, spans, launches = quant_workload(args, dev)
            gbs = (3 * M * K + 4 * M) / (ms * 1e-3) / 1e9
            line = {"metric": f"{'GELU ' if args.act == 'gelu' else ''}activation quantiser GB/s", "value": round(gbs, 1),
                    "unit": "GB/s", "ms_per_step": round(ms, 4), "n_gpus": 1, "steps": args.steps,
                    "warmup": args.warmup, "higher_is_better": True, "dtype": "bf16->int8",
                    "config": {"workload": "quant", "M": M, "K": K, "act": args.act,
                               "l2": "input larger than L2 (no flush)"},
                    "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                                 "frac": round(gbs / pk["hbm_gbs"], 4), "traffic": None,
                                 "peak_source": f"{pk_src} HBM copy bandwidth"},
                    "clocks": clocks, "gpu_launches": int(round(launches * args.steps)),
                    "breakdown": breakdown(spans, pk)}
        elif args.workload == "qkv_a2a":
            M, ms, clocks, spans, launches = qkv_a2a_workload(args, dev)
            ops = 2 * M * 3 * 5120 * 5120
            ga = spans["gemm_a2a"]
            peak = 2.0 * pk["bf16_tflops"]
            ach = ga["work"] / (ga["ms"] * 1e-3) / 1e12
            line = {"metric": "qkv INT8 GEMM with the exchange in its epilogue, TOPS",
                    "value": round(ops / (ms * 1e-3) / 1e12, 1),
                    "unit": "TOPS", "ms_per_step": round(ms, 4), "n_gpus": 1, "steps": args.steps,
                    "warmup": args.warmup, "higher_is_better": True, "dtype": "int8",
                    "config": {"workload": "qkv_a2a", "M": M, "N": 3 * 5120, "K": 5120, "peers_emulated": args.peers,
                               "qk_norm": args.qknorm,
                               "l2": "256 MB flush per step"},
                    "roofline": {"kernel": "gemm_i8_pair_kernel<false, SCATTER> (tcgen05 cta_group::2 kind::i8 + "
                                           "scatter epilogue)", "bound": "tensor", "achieved": round(ach, 1),
                                 "peak": round(peak, 1), "unit": "TOPS", "frac": round(ach / peak, 4),
                                 "traffic": None},
                    "clocks": clocks, "gpu_launches": int(round(launches * args.steps)),
                    "breakdown": breakdown(spans, pk)}
        elif args.workload == "fused":
            ms, clocks, spans, launches = fused_workload(args, dev)
            line = {"metric": "fused adaLN chain (config 1) ms/step", "value": round(ms, 4), "unit": "ms/step",
                    "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "higher_is_better": False,
                    "dtype": "bf16", "config": {"workload": "fused", "S": args.rows or 32768, "D": 5120},
                    "clocks": clocks, "gpu_launches": int(round(launches * args.steps)),
                    "breakdown": breakdown(spans, pk)}
        else:
            if world < 2:
                raise SystemExit("the a2a workload needs --gpus >= 2")
            S, ms, clocks, spans, launches = a2a_workload(args, rank, world, dev)
            buf = S // world * 40 * 128 * 2
            bus = 4 * buf * (world - 1) / world / (ms * 1e-3) / 1e9
            line = {"metric": "Ulysses a2a bus GB/s (q,k,v forward + inverse)", "value": round(bus, 1),
                    "unit": "GB/s", "ms_per_step": round(ms, 4), "n_gpus": world, "steps": args.steps,
                    "warmup": args.warmup, "higher_is_better": True, "dtype": "bf16",
                    "config": {"workload": "a2a", "S": S, "heads": 40, "head_dim": 128, "exchange": args.exchange},
                    "clocks": clocks, "gpu_launches": int(round(launches * args.steps)),
                    "breakdown": breakdown(spans, pk)}
        if rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1 and dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
