"""Benchmark of the joint-attention forward + backward on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c2|c3|c4|c5] [--impl ours|reference]
                    [--ncu-case]

A step is one forward + backward of the op (axial RoPE inside) over one
synthetic batch of the named configuration, inputs resident in HBM. The
default workload is C2 on one GPU and C5 (below) on N > 1 GPUs (launched under
torch.distributed.run, one rank per GPU); `--config c2` with N > 1 gives every
rank its own C2 problem with no collective on the data path (weak scaling).
The timed region is bracketed by a barrier and a device synchronise, and the
maximum time over ranks is reported. `--config c4` splits
its batch of 8 sequences over the ranks instead (strong scaling, still no
cross-GPU traffic). `--config c5` runs
the long-sequence case sequence-parallel instead: one sequence of 16896 rows
sharded over the ranks (strong scaling); the K/V shards and the dK/dV
contributions cross NVLink through peer memory (`--transport peer`, the
default: copy-engine pulls, stores from the backward's epilogue, device
barriers), or an NCCL send/recv ring (`--transport nccl`); or (`--transport
heads`) two NCCL all-to-alls per pass turn the sequence shards into head
groups, and each rank runs the single-GPU op on its H/N heads over the whole
sequence (foundry_trainer_b200/heads.py).

Rank 0 prints one JSON line: the metric (TFLOP/s, FlashAttention accounting
14*B*H*S^2*D), the roofline of the dominant kernel (the backward kernel,
timed live with CUDA events around its own launches), the end-to-end number
through the public API with host buffers, the CPU baseline (the oracle port
on the host cores, a bounded sample), and the SM clocks seen while timing.

`--impl reference` times the reference's arithmetic on the host cores instead:
the reference's Candle code cannot be built here (no Rust toolchain), so the
CPU restatement in oracle/ stands in for it, on a bounded sample per step.
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
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "joint-attn fwd+bwd TFLOP/s (bf16, FlashAttention accounting 14*B*H*S^2*D)"
UNIT = "TFLOP/s"


def _env_int(name, default):
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"bf16": d.get("bf16_tflops"), "bf16_sustained": d.get("bf16_tflops_sustained"),
                "hbm": d.get("hbm_gbs"), "source": "measured"}
    return {"bf16": 1590.0, "bf16_sustained": 1400.0, "hbm": 6650.0, "source": "fallback"}


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while timing."""

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.dev = device_index
        self.proc = None
        self.lines: list[str] = []
        self._t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.dev)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except (OSError, ValueError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.time(), line.strip()))

    def stop(self, t0: float, t1: float):
        """Summary of the samples taken while the timed region [t0, t1] ran
        (wall clock); a short region that no sample fell into is widened to
        the nearest samples around it, which were taken under the same load."""
        if self.proc is None:
            return None
        time.sleep(0.25)  # let a sample after the region arrive
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self._t is not None:
            self._t.join(timeout=2)
        rows = []
        for ts, ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 10:
                continue
            try:
                rows.append((ts, float(parts[2]), float(parts[3]), parts[6:10]))
            except ValueError:
                continue
        inside = [r for r in rows if t0 <= r[0] <= t1]
        if not inside and rows:
            rows.sort(key=lambda r: min(abs(r[0] - t0), abs(r[0] - t1)))
            inside = rows[:2]
        if not inside:
            return None
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = set()
        for r in inside:
            for n, val in zip(names, r[3]):
                if val.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(r[1] for r in inside), "sm_max_mhz": inside[0][2],
                "reasons": sorted(reasons), "samples": len(inside),
                "window": "timed region" if any(t0 <= r[0] <= t1 for r in inside)
                          else "nearest samples around the timed region"}


# ------------------------------------------------------------- CPU oracle
def cpu_oracle_sample(cfg, budget_s: float = 12.0, min_heads: int = 1):
    """Times the oracle port (numpy fp32) on whole heads of the workload until
    about `budget_s` seconds of CPU work; returns (TFLOP/s, heads, seconds)."""
    import numpy as np

    from foundry_trainer_b200 import configs
    from oracle import attn_oracle as orc
    q, k, v, d_o = configs.make_inputs(cfg, batch=1)
    pos = configs.positions(cfg.txt, cfg.grid).numpy()
    qn, kn, vn, dn = (t.float().numpy() for t in (q, k, v, d_o))
    heads, t0 = 0, time.perf_counter()
    while heads < cfg.H and (heads < min_heads or time.perf_counter() - t0 < budget_s):
        orc.attn_fwd_bwd_bshd(qn, kn, vn, dn, "f32", heads=[heads], rope_pos=pos)
        heads += 1
    dt = time.perf_counter() - t0
    flops = 14.0 * heads * cfg.S * cfg.S * cfg.D
    return flops / dt / 1e12, heads, dt, np.__version__


def _oracle_rows_step(orc, qn, kn, vn, dn, pos, rows):
    """One fp32 oracle fwd+bwd of one head for query rows [0, rows) against
    every key (the reference's op graph, lib.rs:133-263, with the axial RoPE
    of lib.rs:77-129 on q and k); returns its FLOPs, 14 * rows * S * D."""
    cos, sin = orc.rope_tables(pos, "f32")
    qr = orc.apply_rope(qn[:rows], cos[:rows], sin[:rows], "f32")
    kr = orc.apply_rope(kn, cos, sin, "f32")
    orc.attn_fwd(qr, kr, vn, "f32", return_lse=True)
    dq, dk, dv = orc.attn_bwd(qr, kr, vn, dn[:rows], "f32")
    orc.apply_rope_grad(dq, cos[:rows], sin[:rows], "f32")
    orc.apply_rope_grad(dk, cos, sin, "f32")
    return 14.0 * rows * kn.shape[0] * kn.shape[2]


def run_reference(args, cfg, rank):
    """The reference arm: the oracle port on the host cores, rank 0 only.
    A step is one head of the workload: the whole head when it is short
    (C1, C2, C4 per sequence), else (C5) the query rows of one 2112-row
    shard against all 16896 keys, so the run stays within a few minutes."""
    if rank != 0:
        return
    from foundry_trainer_b200 import configs
    from oracle import attn_oracle as orc
    q, k, v, d_o = configs.make_inputs(cfg, batch=1)
    pos = configs.positions(cfg.txt, cfg.grid).numpy()
    qn, kn, vn, dn = (t[0, :, :1].float().numpy() for t in (q, k, v, d_o))  # head 0 (S, 1, D)
    rows = cfg.S if cfg.S <= 8192 else cfg.S // 8
    for _ in range(args.warmup):
        _oracle_rows_step(orc, qn, kn, vn, dn, pos, rows)
    t0 = time.perf_counter()
    flops = 0.0
    for _ in range(args.steps):
        flops += _oracle_rows_step(orc, qn, kn, vn, dn, pos, rows)
    dt = time.perf_counter() - t0
    value = flops / dt / 1e12
    cores = os.cpu_count()
    what = (f"1 of {cfg.H} heads" if rows == cfg.S else
            f"query rows 0-{rows - 1} (one of {cfg.S // rows} shards) of 1 of {cfg.H} heads "
            f"against all {cfg.S} keys")
    sample = (f"{what} of {cfg.name} (B=1, S={cfg.S}, D={cfg.D}) fwd+bwd per step, "
              f"fp32 numpy restatement of lib.rs:133-263 with RoPE (Candle CPU build unavailable: "
              f"no Rust toolchain)")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt * 1000.0 / args.steps, "higher_is_better": True,
        "scaling": "strong" if cfg.name in ("c4", "c5") else "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded, configs.make_inputs)",
        "config": {"workload": cfg.name, "B": cfg.B, "H": cfg.H, "S": cfg.S, "D": cfg.D,
                   "txt": cfg.txt, "img_grid": cfg.grid, "rope": "axial (t,h,w,l), theta 10000"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------- C3: LoRA block
def cpu_block_sample(txt_len=512, grid=64, dim=3072, heads=24, rank_lora=16, head_chunk=4):
    """One C3 LoRA step on the host cores: the block code of blocks.py in
    fp32 torch, its joint attention and q/k prologue from the oracle port
    (numpy, `head_chunk` heads at a time). Returns (steps/s, seconds)."""
    import numpy as np
    import torch

    from foundry_trainer_b200 import blocks
    from oracle import attn_oracle as orc

    pos = blocks.joint_positions(txt_len, grid).numpy()
    eps = blocks.NORM_EPS

    def chunks(H):
        return [list(range(i, min(i + head_chunk, H))) for i in range(0, H, head_chunk)]

    class _OracleJoint(torch.autograd.Function):
        @staticmethod
        def forward(ctx, q_t, k_t, v_t, q_i, k_i, v_i, wq_t, wk_t, wq_i, wk_i):
            T = q_t.shape[1]
            n = lambda t: t[0].detach().numpy()
            ins = [n(x) for x in (q_t, k_t, v_t, q_i, k_i, v_i)]
            ws = [x.detach().numpy() for x in (wq_t, wk_t, wq_i, wk_i)]
            q = np.concatenate([orc.qk_norm_rope(ins[0], ws[0], eps, pos[:T], "f32"),
                                orc.qk_norm_rope(ins[3], ws[2], eps, pos[T:], "f32")], 0)
            k = np.concatenate([orc.qk_norm_rope(ins[1], ws[1], eps, pos[:T], "f32"),
                                orc.qk_norm_rope(ins[4], ws[3], eps, pos[T:], "f32")], 0)
            v = np.concatenate([ins[2], ins[5]], 0)
            o = np.concatenate([orc.attn_fwd(q[:, hs], k[:, hs], v[:, hs], "f32")
                                for hs in chunks(q.shape[1])], 1)
            ctx.np = (ins, ws, q, k, v, T)
            return torch.from_numpy(o[:T])[None], torch.from_numpy(o[T:])[None]

        @staticmethod
        def backward(ctx, do_t, do_i):
            ins, ws, q, k, v, T = ctx.np
            d_o = np.concatenate([do_t[0].numpy(), do_i[0].numpy()], 0)
            parts = [orc.attn_bwd(q[:, hs], k[:, hs], v[:, hs], d_o[:, hs], "f32")
                     for hs in chunks(q.shape[1])]
            dq, dk, dv = (np.concatenate([p[j] for p in parts], 1) for j in range(3))
            dq_t, dwq_t = orc.qk_norm_rope_grad(ins[0], ws[0], eps, pos[:T], dq[:T], "f32")
            dq_i, dwq_i = orc.qk_norm_rope_grad(ins[3], ws[2], eps, pos[T:], dq[T:], "f32")
            dk_t, dwk_t = orc.qk_norm_rope_grad(ins[1], ws[1], eps, pos[:T], dk[:T], "f32")
            dk_i, dwk_i = orc.qk_norm_rope_grad(ins[4], ws[3], eps, pos[T:], dk[T:], "f32")
            t = lambda a: torch.from_numpy(np.ascontiguousarray(a))[None]
            w_ = lambda a: torch.from_numpy(np.ascontiguousarray(a))
            return (t(dq_t), t(dk_t), t(dv[:T]), t(dq_i), t(dk_i), t(dv[T:]), w_(dwq_t),
                    w_(dwk_t), w_(dwq_i), w_(dwk_i))

    torch.set_num_threads(os.cpu_count() or 1)
    w = blocks.make_c3_weights(dim, heads, rank_lora, seed=0, dtype=torch.float32)
    g = torch.Generator().manual_seed(1)
    img, txt = torch.randn(1, grid * grid, dim, generator=g), torch.randn(1, txt_len, dim,
                                                                          generator=g)
    temb = torch.randn(dim, generator=g)
    t_img, t_txt = torch.randn(1, grid * grid, dim, generator=g), torch.randn(1, txt_len, dim,
                                                                              generator=g)
    tr = blocks.LoraTrainer(w, blocks.BlockShape(dim, heads), torch.from_numpy(pos),
                            attention=_OracleJoint.apply)
    t0 = time.perf_counter()
    loss = tr.step(img, txt, temb, t_img, t_txt)
    dt = time.perf_counter() - t0
    if not torch.isfinite(loss):
        raise RuntimeError("cpu block sample: non-finite loss")
    return 1.0 / dt, dt


C3_METRIC = "LoRA train steps/s (C3 double-stream block: fwd + bwd to the LoRA factors + AdamW)"


def run_block(args, rank, world, local):
    """C3: one FLUX-style double-stream block (dim 3072, 24 x 128 heads, 512
    text + 64x64 image tokens, 4x GELU MLPs, per-stream adaLN), rank-16
    LoRA (alpha 16) on q/k/v/out of both streams, bf16, random-init weights
    (blocks.make_c3_weights). A step is forward, MSE loss against seeded
    targets, backward to the LoRA factors only, and AdamW; with N ranks each
    runs a replica on its own seeded batch and the LoRA gradients are
    averaged with one NCCL all-reduce per step (weak scaling; `value` counts
    every replica's steps)."""
    if args.impl == "reference":
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable":
                              "the reference's block step is Candle (Rust, not buildable here); "
                              "its CPU arithmetic is timed by --config c2 --impl reference"}),
                  flush=True)
        return
    import torch
    import torch.distributed as dist

    from foundry_trainer_b200 import _lib, blocks, ops
    import ctypes as C

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    dim, heads, rank_lora, txt_len, grid = 3072, 24, 16, 512, 64
    shape = blocks.BlockShape(dim=dim, heads=heads)
    w = blocks.make_c3_weights(dim, heads, rank_lora, seed=0, device=dev)
    g = torch.Generator().manual_seed(1 + rank)
    mk = lambda *sh: torch.randn(*sh, generator=g).to(device=dev, dtype=torch.bfloat16)
    img, txt, temb = mk(1, grid * grid, dim), mk(1, txt_len, dim), mk(dim)
    t_img, t_txt = mk(1, grid * grid, dim), mk(1, txt_len, dim)

    tr = blocks.LoraTrainer(w, shape, blocks.joint_positions(txt_len, grid), lora_scale=1.0,
                            grad_hook=blocks.allreduce_mean if world > 1 else None)
    step = lambda: tr.step(img, txt, temb, t_img, t_txt)
    flush_buf = torch.empty(256 * 1024 * 1024 // 4, device=dev, dtype=torch.float32)
    lib = _lib.load()
    sampler = ClockSampler(local)
    sampler.start()
    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    if ops.device_status() != 0:
        raise RuntimeError("device-side bounded wait expired during warm-up")
    K = args.steps
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    lib.fa_timing_enable(1)
    for kid in (0, 1):
        lib.fa_timing_read(kid, C.byref(C.c_double()), C.byref(C.c_int()))
    t_region0 = time.time()
    for i in range(K):
        flush_buf.zero_()
        starts[i].record()
        loss = step()
        ends[i].record()
    torch.cuda.synchronize()
    t_region1 = time.time()
    lib.fa_timing_enable(0)
    kt = {}
    for kid, name in ((0, "fwd"), (1, "bwd")):
        ms, n = C.c_double(), C.c_int()
        lib.fa_timing_read(kid, C.byref(ms), C.byref(n))
        kt[name] = ms.value / max(n.value, 1)
    if world > 1:
        dist.barrier()
    clocks = sampler.stop(t_region0, t_region1)
    if ops.device_status() != 0:
        raise RuntimeError("device-side bounded wait expired while timing")
    step_ms = sum(a.elapsed_time(b) for a, b in zip(starts, ends))
    t = torch.tensor([step_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    step_ms_max = t.item()

    # end to end: every step's img, txt, temb, targets in from pinned host
    # memory and the loss out
    e2e = None
    if not args.no_e2e:
        host = [x.cpu().pin_memory() for x in (img, txt, temb, t_img, t_txt)]
        dbuf = [torch.empty_like(x) for x in (img, txt, temb, t_img, t_txt)]
        h_loss = torch.empty((), dtype=torch.float32).pin_memory()
        h2d = sum(x.numel() * x.element_size() for x in host)
        for _ in range(2):
            for d_, h_ in zip(dbuf, host):
                d_.copy_(h_, non_blocking=True)
            h_loss.copy_(tr.step(*dbuf), non_blocking=True)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(K):
            for d_, h_ in zip(dbuf, host):
                d_.copy_(h_, non_blocking=True)
            h_loss.copy_(tr.step(*dbuf), non_blocking=True)
        e1.record()
        torch.cuda.synchronize()
        te = torch.tensor([e0.elapsed_time(e1)], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        e2e = {"value": world * K / (te.item() / 1e3), "unit": "steps/s",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4,
               "path": "blocks.LoraTrainer.step with pinned host inputs and the loss read back"}
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        v_cpu, secs = cpu_block_sample()
        cpu = {"value": v_cpu, "unit": "steps/s", "cores": os.cpu_count(), "kind": "port",
               "sample": f"one whole C3 LoRA step (fp32 torch block code, numpy oracle "
                         f"attention and q/k prologue), {secs:.1f} s"}
    peaks = _peaks()
    S = txt_len + grid * grid
    attn_bwd_flops = 10.0 * heads * S * S * 128
    line = {
        "metric": C3_METRIC, "value": world * K / (step_ms_max / 1e3), "unit": "steps/s",
        "n_gpus": world, "steps": K, "warmup": max(args.warmup, 3),
        "ms_per_step": step_ms_max / K, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded: hidden, temb, targets ~ N(0,1); weights ~ N(0,0.02), "
                "LoRA A ~ N(0,1/3072), B = 0)",
        "config": {"workload": f"c3: double-stream block dim {dim}, {heads}x128 heads, "
                               f"{txt_len} text + {grid}x{grid} image tokens, 4x GELU MLP, "
                               f"LoRA r{rank_lora} alpha 16 on q/k/v/out of both streams",
                   "parallelism": f"data-parallel x{world} (LoRA grads all-reduced)",
                   "l2": "flushed between timed steps (256 MB write outside the step events)"},
        "roofline": {"kernel": "attn_bwd_kernel", "bound": "tensor",
                     "achieved": attn_bwd_flops / (kt["bwd"] / 1e3) / 1e12 if kt["bwd"] else None,
                     "peak": peaks["bf16"], "unit": "TFLOP/s",
                     "frac": (attn_bwd_flops / (kt["bwd"] / 1e3) / 1e12 / peaks["bf16"]
                              if kt["bwd"] else None),
                     "traffic": None, "peak_source": f"{peaks['source']} bf16",
                     "fwd_kernel_ms": kt["fwd"], "bwd_kernel_ms": kt["bwd"]},
        "cpu_baseline": cpu,
        "e2e": e2e,
        # per step: q, k prologues + v concat + fwd; dO concat + delta + bwd +
        # dQ finish + q, k prologue backwards
        "gpu_launches": 10 * K,
        "clocks": clocks,
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------- ours
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default=None, choices=["c1", "c2", "c3", "c4", "c5"],
                    help="workload; default c2 on one GPU (BASELINE's headline "
                         "configuration) and c5 on N > 1 (one 16896-row sequence "
                         "sharded over the ranks: the sequence-parallel NVLink path)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--transport", default="peer", choices=["heads", "peer", "nccl"],
                    help="c5 exchange: head groups by NCCL all-to-all (heads), peer memory "
                         "(copy-engine pulls, peer stores, device barriers) or NCCL send/recv "
                         "round a ring")
    ap.add_argument("--peer-copy", default="ce", choices=["ce", "sm"],
                    help="peer transport: K/V pulled by the copy engines (ce) or by a copy "
                         "kernel beside the attention CTAs (sm)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--ncu-case", action="store_true",
                    help="run --warmup eager fwd+bwd steps of --config and exit (no timing): "
                         "the small case ncu captures")
    ap.add_argument("--timeline", action="store_true",
                    help="c5 peer transport: run four eager steps with device events at the "
                         "schedule's milestones and print every rank's milestones of the last "
                         "one (ms since the rank's own step start), then exit")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    rank = _env_int("RANK", 0)
    world = _env_int("WORLD_SIZE", 1)
    local = _env_int("LOCAL_RANK", 0)
    if args.config is None:
        args.config = "c2" if world == 1 else "c5"

    from foundry_trainer_b200 import configs
    cfg = configs.CONFIGS.get(args.config)

    if args.config == "c3":
        run_block(args, rank, world, local)
        return
    if args.impl == "reference":
        run_reference(args, cfg, rank)
        return

    import ctypes as C

    import torch
    import torch.distributed as dist

    from foundry_trainer_b200 import _lib, ops

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)

    ring_mode = cfg.name == "c5"
    batch_mode = cfg.name == "c4"
    b_loc = cfg.B
    pos_full = configs.positions(cfg.txt, cfg.grid)
    if ring_mode:
        # strong scaling: one sequence sharded along S over the ranks, K/V
        # (and dK/dV accumulators) passed round a ring over NCCL
        from foundry_trainer_b200 import ring
        if cfg.S % world != 0:
            raise SystemExit(f"{cfg.name}: S={cfg.S} does not split over {world} ranks")
        n_loc = cfg.S // world
        sl = slice(rank * n_loc, (rank + 1) * n_loc)
        q, k, v, d_o = (t[:, sl].contiguous().to(dev) for t in configs.make_inputs(cfg))
        pos = pos_full[sl].contiguous().to(dev)
        scale = ops.default_scale(cfg.D)
        if args.transport == "peer":
            from foundry_trainer_b200 import peer
            ex = peer.PeerExchange(cfg.B, n_loc, cfg.H, cfg.D, copy=args.peer_copy)
            pkern = peer.PeerKernels()

            def make_step(q, k, v, d_o):
                outs = {}

                def step(trace=None):
                    # the status word is checked around the timed region, not per call
                    o_, lse_, q_r, k_all, v_all = peer.peer_fwd(q, k, v, pos, scale, ex, pkern,
                                                                trace, check_status=False)
                    outs["o"] = o_
                    outs["dq"], outs["dk"], outs["dv"] = peer.peer_bwd(
                        q_r, k_all, v_all, o_, d_o, lse_, pos, scale, ex, pkern, trace,
                        check_status=False)
                return step, outs
        elif args.transport == "heads":
            from foundry_trainer_b200 import heads as hpar
            hex_, hkern = hpar.HeadExchange(), hpar.HeadKernels()
            pos_all = pos_full.contiguous().to(dev)  # every rank attends the whole sequence

            def make_step(q, k, v, d_o):
                outs = {}

                def step():
                    o_, state = hpar.head_fwd(q, k, v, pos_all, scale, hex_, hkern)
                    outs["o"] = o_
                    outs["dq"], outs["dk"], outs["dv"] = hpar.head_bwd(d_o, state, scale, hex_,
                                                                       hkern)
                return step, outs
        else:
            comm, kern = ring.RingComm(), ring.RingKernels()

            def make_step(q, k, v, d_o):
                outs = {}

                def step():
                    o_, lse_, q_r, k_r = ring.ring_fwd(q, k, v, pos, scale, comm, kern)
                    outs["o"] = o_
                    outs["dq"], outs["dk"], outs["dv"] = ring.ring_bwd(q_r, k_r, v, o_, d_o, lse_,
                                                                        pos, scale, comm, kern)
                return step, outs
    else:
        n_loc = cfg.S
        if batch_mode:
            # strong scaling: the B sequences of the batch split over the
            # ranks (B / N each), no cross-GPU traffic
            if cfg.B % world != 0:
                raise SystemExit(f"{cfg.name}: B={cfg.B} does not split over {world} ranks")
            b_loc = cfg.B // world
            bl = slice(rank * b_loc, (rank + 1) * b_loc)
            q, k, v, d_o = (t[bl].contiguous().to(dev) for t in configs.make_inputs(cfg))
        else:
            # weak scaling: each rank owns a whole problem of cfg's size
            q, k, v, d_o = (t.to(dev) for t in configs.make_inputs(cfg))
        pos = pos_full.to(dev)
        rope = ops.Rope(pos)

        def make_step(q, k, v, d_o):
            o = torch.empty_like(q)
            lse = torch.empty((q.shape[0], cfg.H, cfg.S), device=dev, dtype=torch.float32)
            dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
            outs = {"o": o, "dq": dq, "dk": dk, "dv": dv}

            saved = {}

            def step():
                # the backward reuses the forward's rotated q, k (fa_bwd_saved)
                ops.attn_fwd(q, k, v, rope=rope, out=o, lse=lse, saved=saved)
                ops.attn_bwd(q, k, v, o, d_o, lse, rope=rope, dq=dq, dk=dk, dv=dv, saved=saved)
            return step, outs
    step, outs = make_step(q, k, v, d_o)
    flush_buf = torch.empty(256 * 1024 * 1024 // 4, device=dev, dtype=torch.float32)
    lib = _lib.load()

    if args.timeline:
        if not (ring_mode and args.transport == "peer"):
            raise SystemExit("--timeline traces the c5 peer-memory schedule (--config c5)")
        trace: list = []
        for _ in range(4):
            trace.clear()
            if world > 1:
                dist.barrier()
            torch.cuda.synchronize()
            step(trace)
            torch.cuda.synchronize()
        if ops.device_status() != 0:
            raise RuntimeError("device-side bounded wait expired")
        def report(kind):
            t0 = trace[0][1]
            rows = [(name, t0.elapsed_time(e)) for name, e in trace]
            allrows = [rows]
            if world > 1:
                allrows = [None] * world
                dist.all_gather_object(allrows, rows)
            if rank == 0:
                for r, rr in enumerate(allrows):
                    print(f"{kind} rank {r}: " + " ".join(f"{nm}={t:.3f}" for nm, t in rr),
                          flush=True)
        report("eager")
        # the same schedule captured in a CUDA graph, as the timed step runs it
        # (the events become record nodes; the last replay's times are read)
        trace.clear()
        g_tl = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_tl):
            step(trace)
        for _ in range(4):
            if world > 1:
                dist.barrier()
            torch.cuda.synchronize()
            g_tl.replay()
            torch.cuda.synchronize()
        if ops.device_status() != 0:
            raise RuntimeError("device-side bounded wait expired")
        report("graph")
        del g_tl
        ex.close()
        if world > 1:
            dist.destroy_process_group()
        return

    if args.ncu_case:
        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize()
        if ops.device_status() != 0:
            raise RuntimeError("device-side bounded wait expired")
        print("ncu case ok", flush=True)
        if ring_mode and args.transport == "peer":
            ex.close()
        if world > 1:
            dist.destroy_process_group()
        return

    sampler = ClockSampler(local)
    sampler.start()  # started early so samples exist under load near the timed region
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if ops.device_status() != 0:
        raise RuntimeError("device-side bounded wait expired during warm-up")
    # The timed step replays a CUDA graph of the same public-API calls, so
    # host-side launch overhead (ctypes, descriptor encoding) is not timed as
    # device idle; per-kernel times come from an eager pass with the event hooks.
    # The NCCL ring and head-group steps hold NCCL exchanges and run eagerly;
    # the peer step (copies, device barriers, kernels on three streams) is
    # captured.
    if ring_mode and args.transport in ("nccl", "heads"):
        run = step
    else:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()
        run = graph.replay
    run()
    torch.cuda.synchronize()

    K = args.steps
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    # keep the GPU loaded for ~0.5 s before timing (clocks settle, and the
    # sampler sees the load); these replays are not timed
    t_end = time.time() + 0.5
    while time.time() < t_end:
        run()
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t_region0 = time.time()
    wall0 = time.perf_counter()
    for i in range(K):
        flush_buf.zero_()  # L2 (126 MB) flushed between timed steps, outside the events
        starts[i].record()
        run()
        ends[i].record()
    torch.cuda.synchronize()
    wall = time.perf_counter() - wall0
    t_region1 = time.time()
    if world > 1:
        dist.barrier()
    clocks = sampler.stop(t_region0, t_region1)
    # per-kernel device time: eager steps with the library's event hooks
    lib.fa_timing_enable(1)
    for kid in (0, 1):  # drop anything recorded before
        lib.fa_timing_read(kid, C.byref(C.c_double()), C.byref(C.c_int()))
    for i in range(K):
        flush_buf.zero_()
        step()
    torch.cuda.synchronize()
    lib.fa_timing_enable(0)
    kt = {}
    for kid, name in ((0, "fwd"), (1, "bwd")):
        ms, n = C.c_double(), C.c_int()
        _lib.check(lib.fa_timing_read(kid, C.byref(ms), C.byref(n)), "fa_timing_read")
        kt[name] = (ms.value, n.value)
    if ops.device_status() != 0:
        raise RuntimeError("device-side bounded wait expired while timing")
    step_ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends))
    t = torch.tensor([step_ms, kt["bwd"][0] / max(kt["bwd"][1], 1),
                      kt["fwd"][0] / max(kt["fwd"][1], 1)], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    step_ms_max, bwd_ms, fwd_ms = t.tolist()

    # whole-job FLOPs per step: every rank's own problem (weak), or the one
    # sharded sequence or batch (ring / batch split, strong)
    strong = ring_mode or batch_mode
    flops_step = cfg.flops_fwd_bwd() * (1 if strong else world)
    value = K * flops_step / (step_ms_max / 1e3) / 1e12
    # per kernel launch: the whole local problem, or one ring block
    blk = 4.0 * b_loc * cfg.H * n_loc * n_loc * cfg.D

    peaks = _peaks()
    timed_seconds = step_ms_max / 1e3
    peak_kind = "bf16_sustained" if timed_seconds > 2.0 else "bf16"
    peak = peaks[peak_kind]
    # the peer path's backward is one launch over all W shards' keys
    # (as is the head-group backward: all S rows, H / W heads)
    bwd_flops = 2.5 * blk * (world if ring_mode and args.transport in ("peer", "heads") else 1)
    achieved = bwd_flops / (bwd_ms / 1e3) / 1e12
    traffic = None
    tf = ROOT / "profiles" / "traffic.json"
    if tf.exists():
        try:
            traffic = json.loads(tf.read_text()).get(cfg.name, {}).get("attn_bwd_kernel")
        except (ValueError, AttributeError):
            traffic = None
    roofline = {"kernel": "attn_bwd_kernel", "bound": "tensor", "achieved": achieved,
                "peak": peak, "unit": UNIT, "frac": achieved / peak, "traffic": traffic,
                "peak_source": f"{peaks['source']} {peak_kind}",
                "fwd_kernel": {"achieved": blk / (fwd_ms / 1e3) / 1e12,
                               "ms": fwd_ms},
                "bwd_kernel_ms": bwd_ms,
                "flops_per_launch": bwd_flops}

    # ---- secondary: the same step with the deterministic backward
    # (fa_bwd deterministic=1: identical bits across repeats), same timing
    det = None
    if not ring_mode:
        o_d, lse_d = torch.empty_like(q), torch.empty((q.shape[0], cfg.H, cfg.S), device=dev)
        dq_d, dk_d, dv_d = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)

        def det_step():
            ops.attn_fwd(q, k, v, rope=rope, out=o_d, lse=lse_d)
            ops.attn_bwd(q, k, v, o_d, d_o, lse_d, rope=rope, dq=dq_d, dk=dk_d, dv=dv_d,
                         deterministic=True)
        for _ in range(args.warmup):
            det_step()
        g_det = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_det):
            det_step()
        g_det.replay()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        ds_, de_ = ([torch.cuda.Event(enable_timing=True) for _ in range(K)] for _ in range(2))
        for i in range(K):
            flush_buf.zero_()
            ds_[i].record()
            g_det.replay()
            de_[i].record()
        torch.cuda.synchronize()
        td = torch.tensor([sum(a.elapsed_time(b) for a, b in zip(ds_, de_))], device=dev,
                          dtype=torch.float64)
        if world > 1:
            dist.all_reduce(td, op=dist.ReduceOp.MAX)
        det = {"value": K * flops_step / (td.item() / 1e3) / 1e12, "unit": UNIT,
               "ms_per_step": td.item() / K,
               "what": "the same step with fa_bwd deterministic=1 (bit-identical repeats: each "
                       "128-key tile's dQ contribution stored in its own fp32 slot, summed in "
                       "slot order by the finish pass; no fa_bwd_saved reuse)"}
        del g_det
        if ops.device_status() != 0:
            raise RuntimeError("device-side bounded wait expired (deterministic step)")

    # ---- end to end through the public API with host buffers
    e2e = None
    if not args.no_e2e:
        # End to end through the public API: every step copies its own q, k,
        # v, dO in from pinned host memory and its o, dq, dk, dv out. Two sets
        # of device buffers and three streams: step i+1's host->device copies
        # and step i-1's device->host copies run while step i computes.
        names = ("o", "dq", "dk", "dv")
        sets = []
        for _ in range(2):
            ins = [torch.empty_like(x) for x in (q, k, v, d_o)]
            run_s, outs_s = make_step(*ins)
            sets.append((ins, run_s, outs_s))
        hin = [x.cpu().pin_memory() for x in (q, k, v, d_o)]
        hout = [torch.empty_like(outs[n], device="cpu").pin_memory() for n in names]
        h2d = sum(x.numel() * x.element_size() for x in hin)
        d2h = sum(x.numel() * x.element_size() for x in hout)
        s_in, s_cmp, s_out = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()
        ev_in = [torch.cuda.Event() for _ in range(2)]
        ev_cmp = [torch.cuda.Event() for _ in range(2)]
        ev_out = [torch.cuda.Event() for _ in range(2)]

        def pipeline(n):
            for i in range(n + 2):
                if i < n:  # inputs of step i into set i % 2 (free once step i-2 computed)
                    si = i % 2
                    with torch.cuda.stream(s_in):
                        if i >= 2:
                            s_in.wait_event(ev_cmp[si])
                        for dst, src in zip(sets[si][0], hin):
                            dst.copy_(src, non_blocking=True)
                        ev_in[si].record(s_in)
                j = i - 1
                if 0 <= j < n:  # step j (its outputs' set free once step j-2 was read out)
                    sj = j % 2
                    with torch.cuda.stream(s_cmp):
                        s_cmp.wait_event(ev_in[sj])
                        if j >= 2:
                            s_cmp.wait_event(ev_out[sj])
                        sets[sj][1]()
                        ev_cmp[sj].record(s_cmp)
                m = i - 2
                if 0 <= m < n:  # results of step m out to the host
                    sm = m % 2
                    with torch.cuda.stream(s_out):
                        s_out.wait_event(ev_cmp[sm])
                        for dst, name in zip(hout, names):
                            src = sets[sm][2][name]
                            src.record_stream(s_out)  # (ring outputs are fresh tensors per step)
                            dst.copy_(src, non_blocking=True)
                        ev_out[sm].record(s_out)

        pipeline(args.warmup)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        cur = torch.cuda.current_stream()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record(cur)
        for st_ in (s_in, s_cmp, s_out):
            st_.wait_event(s0)
        pipeline(K)
        for st_ in (s_in, s_cmp, s_out):
            cur.wait_stream(st_)
        s1.record(cur)
        torch.cuda.synchronize()
        te = torch.tensor([s0.elapsed_time(s1)], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        e2e = {"value": K * flops_step / (te.item() / 1e3) / 1e12, "unit": UNIT,
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "ms_per_step": te.item() / K,
               "path": ("ring.ring_fwd + ring.ring_bwd (C ABI fa_fwd_partial/fa_bwd_partial "
                        "round an NCCL ring)" if ring_mode and args.transport == "nccl" else
                        "heads.head_fwd + heads.head_bwd (NCCL all-to-alls; C ABI fa_fwd/"
                        "fa_bwd_saved on H/W heads)" if ring_mode and args.transport == "heads"
                        else
                        "peer.peer_fwd + peer.peer_bwd (C ABI fa_fwd_fold/fa_merge_f32/"
                        "fa_bwd_scatter/fa_reduce_cast_f32 over peer memory)" if ring_mode else
                        "ops.attn_fwd + ops.attn_bwd (C ABI fa_fwd/fa_bwd_saved)") +
                       " per rank; every step copies its pinned host q,k,v,dO in and o,dq,dk,dv "
                       "out; copies of the neighbouring steps overlap the compute on separate "
                       "streams (the timed region covers all K steps' copies and compute)"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v_cpu, heads, secs, _ = cpu_oracle_sample(cfg)
        cpu = {"value": v_cpu, "unit": UNIT, "cores": os.cpu_count(), "kind": "port",
               "sample": f"{heads} of {cfg.H} heads of {cfg.name} fwd+bwd with RoPE, fp32 numpy "
                         f"oracle, {secs:.1f} s"}

    if ring_mode and args.transport == "peer":
        ex.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    if ring_mode and args.transport == "peer":
        # fwd: rope q, rope k, the fold launches (+ merge and barrier, and
        # with the copy kernel 2 per pulled shard, when W > 1); bwd: prepare,
        # one scatter launch, reduce-cast, dQ cast (+ barrier)
        n_folds = len(peer.fold_groups(world))
        launches_per_step = (2 + n_folds + 4 + (3 if world > 1 else 0) +
                             (2 * (world - 1) if args.peer_copy == "sm" else 0))
        workload = (f"{cfg.name}: B={cfg.B} H={cfg.H} S={cfg.S} ({cfg.txt} text + "
                    f"{cfg.grid}x{cfg.grid} image) D={cfg.D}, one sequence sharded "
                    f"{n_loc} rows per rank, non-causal, axial RoPE")
        parallelism = (f"sequence-parallel x{world} over peer memory (K/V pulled by "
                       f"{'a copy kernel' if args.peer_copy == 'sm' else 'the copy engines'}, "
                       f"dK/dV rows stored into the owners by the backward's epilogue)")
    elif ring_mode and args.transport == "heads":
        # fwd: table + fwd kernel; bwd: delta + bwd kernel + dQ finish (the
        # all-to-alls are NCCL's kernels, not counted)
        launches_per_step = 5
        workload = (f"{cfg.name}: B={cfg.B} H={cfg.H} S={cfg.S} ({cfg.txt} text + "
                    f"{cfg.grid}x{cfg.grid} image) D={cfg.D}, one sequence sharded "
                    f"{n_loc} rows per rank, non-causal, axial RoPE inside the op")
        parallelism = (f"head groups x{world}: NCCL all-to-all of q,k,v / O / dO / dq,dk,dv "
                       f"between the sequence shards and {cfg.H // world} heads per rank over "
                       f"the whole sequence")
    elif ring_mode:
        # fwd: rope q, rope k, W blocks + W merges, O cast; bwd: prepare,
        # W blocks, W-1 accumulator adds, 3 casts
        launches_per_step = 4 * world + 6
        workload = (f"{cfg.name}: B={cfg.B} H={cfg.H} S={cfg.S} ({cfg.txt} text + "
                    f"{cfg.grid}x{cfg.grid} image) D={cfg.D}, one sequence sharded "
                    f"{n_loc} rows per rank, non-causal, axial RoPE")
        parallelism = f"sequence ring x{world} (NCCL send/recv of K,V and fp32 dK,dV)"
    else:
        # (cos, sin) table + fwd (q, k rotated in its tile loads); delta (+ dQ
        # clear) + bwd + dQ finish
        launches_per_step = 5
        if batch_mode:
            workload = (f"{cfg.name}: B={cfg.B} H={cfg.H} S={cfg.S} "
                        f"({cfg.txt} text + {cfg.grid}x{cfg.grid} image) D={cfg.D}, the batch "
                        f"split {b_loc} sequences per rank, non-causal, axial RoPE inside the op")
            parallelism = f"batch split x{world} (B={b_loc} per rank), no collective"
        else:
            workload = (f"{cfg.name}: B={cfg.B} H={cfg.H} S={cfg.S} "
                        f"({cfg.txt} text + {cfg.grid}x{cfg.grid} image) D={cfg.D} "
                        f"per rank, non-causal, axial RoPE inside the op")
            parallelism = f"batch-sharded x{world}, no collective on the data path"
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": K,
        "warmup": args.warmup, "ms_per_step": step_ms_max / K, "higher_is_better": True,
        "scaling": "strong" if strong else "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded torch.Generator, q,k,v ~ 0.5*N(0,1), dO ~ N(0,1))",
        "config": {"workload": workload,
                   "per_rank_B": b_loc, "H": cfg.H, "S": cfg.S, "S_per_rank": n_loc, "D": cfg.D,
                   "l2": "flushed between timed steps (256 MB write outside the step events)",
                   "parallelism": parallelism},
        "roofline": roofline,
        "cpu_baseline": cpu,
        "e2e": e2e,
        "gpu_launches": launches_per_step * K,
        "clocks": clocks,
        "wall_s_timed": wall,
        "deterministic": det,
    }
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
