#!/usr/bin/env python
"""Benchmark of the Ulysses context-parallel attention layer (the path's headline metric).

A step is one layer: the fused first stage (RoPE/RMSNorm + transposition into per-peer blocks),
the seq->head crossing of Q/K/V (NCCL all-to-all; none at degree 1), the sm_100a attention
kernel, the head->seq crossing of O and the landing. Inputs are synthetic, seeded, resident in
HBM before the timed region and larger than L2 (126 MB), so no flush is needed between steps.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c2|c3|c5] [--impl reference]

Under torchrun (N > 1) every rank holds its `torch.tensor_split` rows; the step time is the max
over ranks of CUDA-event time. Rank 0 prints one JSON line.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

METRIC = "CP attention layer ms and TFLOP/s at 1/2/4/8 B200 (device-timed, max over ranks)"
FALLBACK_BF16_TFLOPS = 1590.0

CONFIGS = {
    "c2": {
        "workload": "C2 video-DiT joint self-attention: B=1 H=24 D=128 S=21x30x52+512=33272, "
        "non-causal, 3D axial RoPE (44/42/42) on the video tokens, inputs N(0,1)*0.5",
        "batch": 1, "heads": 24, "heads_kv": 24, "dim": 128, "seq": 33272, "causal": False,
        "rope": ("axial", (21, 30, 52), (44, 42, 42), 10000.0, 0, 512), "norm": False, "amp": 0.5,
    },
    "c3": {
        "workload": "C3 Flux-style joint attention: B=2 H=24 D=128 S=512+64x64=4608, non-causal, "
        "per-head RMSNorm on Q,K then 2D axial RoPE (16/56/56, theta 10000)",
        "batch": 2, "heads": 24, "heads_kv": 24, "dim": 128, "seq": 4608, "causal": False,
        "rope": ("axial", (1, 64, 64), (16, 56, 56), 10000.0, 512, 0), "norm": True, "amp": 1.0,
    },
    "c4": {
        "workload": "C4 FP8 video attention: B=1 H=40 D=128 S=21x45x80=75600, non-causal; Q/K "
        "e4m3 with one scale per 64-token x head block (Hadamard turn, K less its global mean), "
        "V e4m3 per-channel scales, P e4m3, fp32 softmax/accumulation; N(0,1), 1% of K x8",
        "batch": 1, "heads": 40, "heads_kv": 40, "dim": 128, "seq": 75600, "causal": False,
        "rope": None, "norm": False, "amp": 1.0, "fp8": True, "k_outliers": 0.01,
    },
    "c5": {
        "workload": "C5 causal GQA prefill: B=1 Hq=32 Hkv=8 D=128 S=131071, causal, "
        "1D RoPE theta 500000",
        "batch": 1, "heads": 32, "heads_kv": 8, "dim": 128, "seq": 131071, "causal": True,
        "rope": ("llama", 500000.0), "norm": False, "amp": 1.0,
    },
}


def layer_flops(cfg: dict, heads: int | None = None) -> float:
    """Algorithmic FLOPs (padding excluded): 4·B·H·S²·D, causal 4·B·H·D·S(S+1)/2."""
    b, s, d = cfg["batch"], cfg["seq"], cfg["dim"]
    h = cfg["heads"] if heads is None else heads
    if cfg["causal"]:
        return 4.0 * b * h * d * s * (s + 1) / 2
    return 4.0 * b * h * s * s * d


def make_rope(cfg: dict):
    from cozy_runtime_b200 import rope

    if cfg["rope"] is None:
        return None
    kind = cfg["rope"][0]
    if kind == "axial":
        _, grid, dims, theta, before, after = cfg["rope"]
        return rope.axial(grid, dims, theta, before=before, after=after)
    return rope.llama(cfg["seq"], cfg["dim"], cfg["rope"][1])


#: A kernel is held to the sustained peak (a cuBLAS GEMM looped for seconds under the power cap)
#: only when a single step runs at least this long; shorter steps are held to the burst peak.
SUSTAINED_STEP_S = 1.0


def peaks(fp8: bool = False) -> tuple[float, float, str]:
    """The tensor roofline denominators (burst, sustained) from MEASURED_PEAKS.json, and their
    source. FP8 has no measured figure on this pool: twice the measured bf16 figure (the dense
    e4m3:bf16 ratio of the part), labelled as such."""
    path = ROOT / "MEASURED_PEAKS.json"
    mult, what = (2.0, "2 x ") if fp8 else (1.0, "")
    if path.exists():
        data = json.loads(path.read_text())
        burst = float(data["bf16_tflops"])
        held = float(data.get("bf16_tflops_sustained", burst))
        return mult * burst, mult * held, f"{what}measured bf16 (MEASURED_PEAKS.json)"
    return (mult * FALLBACK_BF16_TFLOPS, mult * FALLBACK_BF16_TFLOPS,
            f"{what}fallback bf16 (MEASURED_PEAKS.json absent)")


class NvmlSampler:
    """SM clock and clock-event reasons read through NVML every 10 ms during the timed region,
    by a thread of rank 0 (read-only queries; no setting is changed). Falls back to
    `ClockSampler` without NVML. Measured at degree 2: sampling from a child process instead
    cost ~3 ms a step (8.9 against 6.0 ms); sampling from every rank's process at degree 8,
    ~0.4 ms."""

    REASONS = (
        ("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
        ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
        ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
        ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"),
    )

    def __init__(self, gpu: int) -> None:
        import threading

        import pynvml

        self.nvml = pynvml
        pynvml.nvmlInit()
        self.handle = pynvml.nvmlDeviceGetHandleByIndex(gpu)
        self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
        self.samples: list[tuple[int, int]] = []
        self.stop = threading.Event()
        self.thread = threading.Thread(target=self._run, daemon=True)

    def _run(self) -> None:
        n = self.nvml
        while not self.stop.is_set():
            try:
                mhz = n.nvmlDeviceGetClockInfo(self.handle, n.NVML_CLOCK_SM)
                reasons = n.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
                self.samples.append((mhz, reasons))
            except n.NVMLError:
                pass
            time.sleep(0.01)

    def __enter__(self):
        self.thread.start()
        return self

    def __exit__(self, *exc):
        self.stop.set()
        self.thread.join(timeout=5)

    def summary(self) -> dict | None:
        if not self.samples:
            return None
        reasons = sorted(
            {name for _, bits in self.samples for name, attr in self.REASONS
             if bits & getattr(self.nvml, attr)}
        )
        return {
            "sm_mhz": statistics.median(s[0] for s in self.samples),
            "sm_max_mhz": self.max_mhz,
            "reasons": reasons,
            "samples": len(self.samples),
            "source": "nvml",
        }


class NullSampler:
    """The other ranks' stand-in: no sampling."""

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return None

    def summary(self) -> None:
        return None


def clock_sampler(gpu: int):
    try:
        return NvmlSampler(gpu)
    except Exception:  # noqa: BLE001 - no NVML: sample through nvidia-smi instead
        return ClockSampler(gpu)


class ClockSampler:
    """nvidia-smi samples of the SM clock and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int) -> None:
        self.gpu, self.proc = gpu, None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.gpu)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True,
            )
        except (FileNotFoundError, OSError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            out, _ = self.proc.communicate(timeout=10)
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self) -> dict | None:
        rows = []
        for ln in getattr(self, "lines", []):
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), parts[5:9]))
            except ValueError:
                continue
        if not rows:
            return None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, flags in rows for i, f in enumerate(flags)
                          if f.lower().startswith("active")})
        return {
            "sm_mhz": statistics.median(r[0] for r in rows),
            "sm_max_mhz": max(r[1] for r in rows),
            "reasons": reasons,
            "samples": len(rows),
        }


def local_gpu_index(local_rank: int) -> int:
    visible = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    if visible:
        ids = [v.strip() for v in visible.split(",") if v.strip()]
        if local_rank < len(ids) and ids[local_rank].isdigit():
            return int(ids[local_rank])
    return local_rank


def cpu_baseline(cfg: dict, budget_s: float = 12.0) -> dict:
    """The reference's CPU computation (torch SDPA math, restated by the oracle) on host cores,
    over a bounded sample of the workload: query-row blocks of one head against the whole
    sequence's keys, repeated until `budget_s`; reported as TFLOP/s of that sample."""
    import torch

    import oracle

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    s, d = cfg["seq"], cfg["dim"]
    rows = 512
    g = torch.Generator().manual_seed(1)
    q = torch.randn(1, rows, 1, d, generator=g).to(torch.bfloat16)
    k = torch.randn(1, s, 1, d, generator=g).to(torch.bfloat16)
    v = torch.randn(1, s, 1, d, generator=g).to(torch.bfloat16)
    # (causal: a block of rows at the sequence's end sees every key, so the same cost)
    flops_call = 4.0 * rows * s * d
    calls, start = 0, time.perf_counter()
    while True:
        oracle.attention_fp32(q, k, v)
        calls += 1
        if time.perf_counter() - start >= budget_s:
            break
    elapsed = time.perf_counter() - start
    return {
        "value": round(flops_call * calls / elapsed / 1e12, 5),
        "unit": "TFLOP/s",
        "cores": threads,
        "kind": "port",
        "sample": f"{calls} calls of 1 head x {rows} query rows x {s} keys x D={d} "
        f"(fp32 math on bf16 inputs, oracle restatement of torch SDPA), {elapsed:.1f} s",
    }


def _reference_rank(rank, world, port, cfg, steps, warmup, threads, sample_seq, outdir):
    """One gloo process of the reference arm: the reference's CPU path for a layer, restated by
    the oracle (`exchange_group`: its collectives included, torch SDPA in bf16 as `compute`),
    on this rank's rows of a sampled layer; writes every step's time (max over ranks)."""
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    import oracle

    torch.set_num_threads(threads)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=timedelta(seconds=900))
    rows = oracle.sequence_rows(sample_seq, world)
    gen = torch.Generator().manual_seed(100 + rank)
    b, d, amp = cfg["batch"], cfg["dim"], cfg["amp"]
    q, k, v = ((torch.randn(b, rows[rank], world, d, generator=gen) * amp).to(torch.bfloat16)
               for _ in range(3))

    def compute(qq, kk, vv):
        return oracle.attention_fp32(qq, kk, vv, causal=cfg["causal"],
                                     dtype=torch.bfloat16).to(torch.bfloat16)

    times = []
    for i in range(warmup + steps):
        dist.barrier()
        began = time.perf_counter()
        oracle.exchange_group(q, k, v, dist.group.WORLD, compute)
        took = torch.tensor([time.perf_counter() - began], dtype=torch.float64)
        dist.all_reduce(took, op=dist.ReduceOp.MAX)
        if i >= warmup:
            times.append(took.item())
    if rank == 0:
        Path(outdir, "times.json").write_text(json.dumps(times))
    dist.destroy_process_group()


def run_reference(args, cfg) -> None:
    """`--impl reference`: the reference's CPU path for this layer (the oracle's restatement of
    its exchange over gloo, torch SDPA as compute) on the box's host cores, as W = --gpus gloo
    processes; rank 0 of a torchrun launch alone runs it. Each step is a bounded sample: one
    head a process over a sequence of at most 8192 tokens (SDPA's rate does not depend on the
    length at these sizes), whole exchanges timed as the max over processes; `value` is the
    sample's TFLOP/s, `ms_per_step` the whole layer's FLOPs at that rate."""
    import socket
    import tempfile

    import torch.multiprocessing as mp

    if int(os.environ.get("RANK", "0")) != 0:
        return
    world = max(1, args.gpus)
    cores = os.cpu_count() or 1
    threads = max(1, cores // world)
    sample_seq = min(cfg["seq"], 8192)
    with socket.socket() as sock:
        sock.bind(("127.0.0.1", 0))
        port = sock.getsockname()[1]
    with tempfile.TemporaryDirectory() as tmp:
        mp.spawn(_reference_rank, args=(world, port, cfg, args.steps, args.warmup, threads,
                                        sample_seq, tmp), nprocs=world, join=True)
        times = json.loads(Path(tmp, "times.json").read_text())
    step_s = statistics.median(times)
    sample = dict(cfg, seq=sample_seq, heads=world, heads_kv=world)
    value = layer_flops(sample) / step_s / 1e12
    flops = layer_flops(cfg)
    kind_note = (f"{world} gloo processes x {threads} threads ({world * threads} of {cores} host "
                 f"threads), one head a process over {sample_seq} tokens (of {cfg['seq']}), "
                 f"the oracle's restatement of the reference's exchange (all-to-all over gloo, "
                 f"torch SDPA in bf16), median of {len(times)} steps of {step_s:.3f} s "
                 f"(max over processes); RoPE/RMSNorm not included")
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": round(value, 5),
        "unit": "TFLOP/s",
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(flops / (value * 1e12) * 1e3, 3) if value else None,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": cfg["workload"], "parallelism": f"gloo{world} (cpu)",
                   "sampled": True},
        "cpu_baseline": {"value": round(value, 5), "unit": "TFLOP/s", "cores": world * threads,
                         "kind": "port", "sample": kind_note},
        "e2e": {"value": round(value, 5), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def first_law_fp32(x, spec, norm: bool, token0: int):
    """The first stage's RMSNorm (unit weight, eps 1e-6) and RoPE in fp32 torch on the GPU: the
    plain PyTorch reference the parity check holds the layer to. x: [B, S, H, D]."""
    import torch

    y = x.float()
    if norm:
        y = y * torch.rsqrt(y.pow(2).mean(-1, keepdim=True) + 1e-6)
    if spec is None:
        return y
    seq, rot = y.shape[1], spec.rotary
    tok = torch.arange(token0, token0 + seq, device=y.device)
    cos, sin = spec.cos.reshape(-1), spec.sin.reshape(-1)
    out = y.clone()
    if spec.interleaved:
        col = torch.arange(rot // 2, device=y.device) * spec.stride_channel
        idx = tok[:, None] * spec.stride_token + col[None, :]
        c, sn = cos[idx][None, :, None, :], sin[idx][None, :, None, :]
        lo, hi = y[..., 0:rot:2], y[..., 1:rot:2]
        out[..., 0:rot:2] = lo * c - hi * sn
        out[..., 1:rot:2] = hi * c + lo * sn
    else:
        half = rot // 2
        col = torch.arange(rot, device=y.device) * spec.stride_channel
        idx = tok[:, None] * spec.stride_token + col[None, :]
        c, sn = cos[idx][None, :, None, :], sin[idx][None, :, None, :]
        lo, hi = y[..., :half], y[..., half:rot]
        out[..., :half] = lo * c[..., :half] - hi * sn[..., :half]
        out[..., half:rot] = hi * c[..., half:] + lo * sn[..., half:]
    return out


def parity_check(q, k, v, out, rows, rank, group, cfg, spec, device, fp8=False) -> dict:
    """One step's output on every rank against fp32 attention computed on that rank's GPU: three
    query heads, up to 512 of this rank's rows (its first and last 256), the keys and values of
    the whole sequence gathered from every rank. The path's bf16 bar: max-abs ≤ 2e-2, mean-abs
    ≤ 2e-3 (max over ranks); FP8: cosine similarity ≥ 0.995 per head (min over heads and
    ranks)."""
    import torch
    import torch.distributed as dist

    heads, hkv = cfg["heads"], cfg["heads_kv"]
    grouping = heads // hkv
    pick = sorted({0, heads // 2, heads - 1})
    kv_pick = sorted({h // grouping for h in pick})
    start, mine = sum(rows[:rank]), rows[rank]
    kx = first_law_fp32(k[:, :, kv_pick], spec, cfg["norm"], start)
    vx = v[:, :, kv_pick].float()
    if group is not None:
        # every rank's rows of these heads (uneven rows: padded to the largest, then cropped)
        most = max(rows)
        pad = torch.zeros(kx.shape[0], most, len(kv_pick), kx.shape[3], device=device)
        kk, vv = pad.clone(), pad.clone()
        kk[:, :mine], vv[:, :mine] = kx, vx
        ks, vs = [torch.empty_like(kk) for _ in rows], [torch.empty_like(vv) for _ in rows]
        dist.all_gather(ks, kk, group=group)
        dist.all_gather(vs, vv, group=group)
        kx = torch.cat([t[:, :n] for t, n in zip(ks, rows, strict=True)], dim=1)
        vx = torch.cat([t[:, :n] for t, n in zip(vs, rows, strict=True)], dim=1)
    sel = torch.arange(mine, device=device)
    if mine > 512:
        sel = torch.cat([sel[:256], sel[-256:]])
    worst, total, count, cos = 0.0, 0.0, 0, 1.0
    for h in pick:
        qx = first_law_fp32(q[:, :, [h]], spec, cfg["norm"], start)[:, sel]
        kvh = kv_pick.index(h // grouping)
        for b in range(q.shape[0]):
            sc = (qx[b, :, 0] @ kx[b, :, kvh].T) / (q.shape[3] ** 0.5)
            if cfg["causal"]:
                cols = torch.arange(kx.shape[1], device=device)
                sc = sc.masked_fill(cols[None, :] > (start + sel)[:, None], float("-inf"))
            want = torch.softmax(sc, dim=-1) @ vx[b, :, kvh]
            got = out[b, sel, h].float()
            err = (got - want).abs()
            worst = max(worst, err.max().item())
            total += err.sum().item()
            count += err.numel()
            cos = min(cos, torch.nn.functional.cosine_similarity(
                got.reshape(1, -1), want.reshape(1, -1)).item())
    stats = torch.tensor([worst, total / max(count, 1), -cos], dtype=torch.float64, device=device)
    if group is not None:
        dist.all_reduce(stats, op=dist.ReduceOp.MAX, group=group)
    worst, mean, neg_cos = stats.tolist()
    ok = -neg_cos >= 0.995 if fp8 else worst <= 2e-2 and mean <= 2e-3
    return {"max_abs": round(worst, 5), "mean_abs": round(mean, 6),
            "min_head_cosine": round(-neg_cos, 6), "ok": bool(ok),
            "bar": "cosine >= 0.995 per head" if fp8 else "max-abs <= 2e-2, mean-abs <= 2e-3",
            "checked": f"heads {pick}, up to 512 rows a rank, vs fp32 torch on the GPU"}


def fp8_first_stage(q, k, v, layout, rank, law, spec, norm, steps, device) -> dict:
    """The FP8 first stage's kernels alone at this rank's shape (statistics, then the e4m3 pack
    into every owner's block, all on this GPU), CUDA events; algorithmic bytes ÷ time."""
    import torch

    from cozy_runtime_b200 import fp8 as fp8_mod

    st = fp8_mod.Fp8Step(q, k, v, layout, rank, rope=spec, norm_q=norm, norm_k=norm, law=law)
    scales = st.scales()  # this rank's statistics: timing only
    b, mine, hq, d = (int(n) for n in q.shape)
    hkv = int(k.shape[2])
    world = layout.world
    u8 = torch.uint8
    codes = [[torch.empty(max(1, mine * b * n[p] * d), dtype=u8, device=device) for p in range(world)]
             for n in (layout.q_n, layout.kv_n, layout.kv_n)]
    sc = [[torch.empty(max(1, b * n[p] * mine), device=device) for p in range(world)]
          for n in (layout.q_n, layout.kv_n)]
    block = law == "block"
    acc = [torch.zeros(b, hkv, d, device=device) for _ in range(2)] if block else [
        torch.zeros(b, n, device=device) for n in (hq, hkv, hkv)]

    def stats():
        if block:
            st.stats_into(*acc)
        else:
            st.head_amax_into(*acc)

    def pack():
        st.pack_to(scales, *([t.data_ptr() for t in c] for c in codes),
                   *([t.data_ptr() for t in c] for c in sc), scale_rows=mine)

    elems = mine * b * d
    read_stats = (2 * hkv if block else hq + 2 * hkv) * elems * 2
    moved_pack = (hq + 2 * hkv) * elems * 3 + (hq + hkv) * mine * b * 4
    out = {"law": law, "rows": mine, "heads": hq}
    for name, fn, nbytes in (("stats", stats, read_stats), ("pack", pack, moved_pack)):
        for _ in range(3):
            fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / steps
        out[f"{name}_us"] = round(ms * 1e3, 1)
        out[f"{name}_gbs"] = round(nbytes / (ms * 1e-3) / 1e9, 1)
    return out


def attention_alone(cfg, layout, rank, steps, device) -> float:
    """ms per launch of this rank's attention with every operand resident (no crossing): the
    same kernel and shapes as inside the layer, on [B, S, heads, D] operands."""
    import torch

    from cozy_runtime_b200 import attention

    qn, kvn = layout.q_n[rank], layout.kv_n[rank]
    if qn == 0:
        return 0.0
    total, b, d = layout.total, cfg["batch"], cfg["dim"]
    gen = torch.Generator(device=device).manual_seed(7)
    q = torch.randn(b, total, qn, d, generator=gen, device=device).to(torch.bfloat16)
    k = torch.randn(b, total, kvn, d, generator=gen, device=device).to(torch.bfloat16)
    v = torch.randn(b, total, kvn, d, generator=gen, device=device).to(torch.bfloat16)
    out = torch.empty_like(q)
    head_map = (layout.group, layout.q_lo[rank], layout.kv_lo[rank])
    for _ in range(2):
        attention.attention_into(out, q, k, v, causal=cfg["causal"], head_map=head_map)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        attention.attention_into(out, q, k, v, causal=cfg["causal"], head_map=head_map)
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def cudnn_attention(cfg, layout, rank, device) -> dict | None:
    """torch SDPA on cuDNN alone (the reference's B200 bf16 row, attention_upstream.py:191-215)
    on this rank's per-GPU shape, CUDA events, 5 launches after 2."""
    import torch
    import torch.nn.functional as F
    from torch.nn.attention import SDPBackend, sdpa_kernel

    qn, total, b, d = layout.q_n[rank], layout.total, cfg["batch"], cfg["dim"]
    if qn == 0:
        return None
    kvn = max(1, qn // layout.group)
    gen = torch.Generator(device=device).manual_seed(9)
    q = torch.randn(b, qn, total, d, generator=gen, device=device).to(torch.bfloat16)
    k = torch.randn(b, kvn, total, d, generator=gen, device=device).to(torch.bfloat16)
    v = torch.randn(b, kvn, total, d, generator=gen, device=device).to(torch.bfloat16)
    try:
        with sdpa_kernel([SDPBackend.CUDNN_ATTENTION]):
            def call():
                return F.scaled_dot_product_attention(q, k, v, is_causal=cfg["causal"],
                                                      enable_gqa=kvn != qn)
            for _ in range(2):
                call()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(5):
                call()
            e1.record()
            torch.cuda.synchronize()
    except Exception as exc:  # noqa: BLE001 - reported, not fatal
        return {"unavailable": str(exc)[:200]}
    ms = e0.elapsed_time(e1) / 5
    return {"ms": round(ms, 4), "tflops": round(layer_flops(cfg, heads=qn) / ms / 1e9, 1),
            "heads": qn, "seq": total, "layout": "[B, H, S, D] contiguous",
            "call": "torch SDPA, SDPBackend.CUDNN_ATTENTION only"}


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=40)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--config", default="c2", choices=sorted(CONFIGS))
    parser.add_argument("--impl", default="cozy", choices=["cozy", "reference"])
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--no-e2e", action="store_true", help="skip the end-to-end leg")
    parser.add_argument("--no-extras", action="store_true",
                        help="skip the parity check, attention-alone, cuDNN and long-run legs")
    parser.add_argument("--long-run-s", type=float, default=0.5,
                        help="after the timed steps, steps until this long has passed (clocks)")
    parser.add_argument("--fp8-law", default="block", choices=["block", "head"],
                        help="FP8 configurations: the 64-token block recipe (c4's) or the "
                        "reference's per-(batch, head) row")
    parser.add_argument("--narrow", action="store_true",
                        help="the int8 wire (exchange(..., narrow=True)); not the headline")
    parser.add_argument("--heads", type=int, default=0,
                        help="profiling only: fewer heads (same sequence and layout)")
    args = parser.parse_args()
    cfg = dict(CONFIGS[args.config])
    if args.heads:
        group = cfg["heads"] // cfg["heads_kv"]
        cfg["heads"], cfg["heads_kv"] = args.heads, max(1, args.heads // group)
        cfg["workload"] += f" [profiling subset: {cfg['heads']} heads]"
    if args.impl == "reference":
        run_reference(args, cfg)
        return

    import torch
    import torch.distributed as dist

    from cozy_runtime_b200 import _lib, attention, ulysses

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    group = None
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", device_id=device, timeout=timedelta(seconds=300))
        group = dist.group.WORLD
    _lib.load()

    batch, heads, hkv, dim, seq = (cfg[k] for k in ("batch", "heads", "heads_kv", "dim", "seq"))
    rows = ulysses.tensor_split_rows(seq, world)
    mine = rows[rank]
    gen = torch.Generator(device=device).manual_seed(1234 + rank)
    amp = cfg["amp"]

    def randn(h):
        return (torch.randn(batch, mine, h, dim, generator=gen, device=device) * amp).to(
            torch.bfloat16)

    q, k, v = randn(heads), randn(hkv), randn(hkv)
    if cfg.get("k_outliers"):
        hit = torch.rand(k.shape, generator=gen, device=device) < cfg["k_outliers"]
        k = torch.where(hit, k * 8, k)
    spec = make_rope(cfg)
    spec = spec.to(device) if spec is not None else None
    norm = ulysses.Norm() if cfg["norm"] else None
    fp8 = bool(cfg.get("fp8"))
    fp8_arg = ("head" if args.fp8_law == "head" else True) if fp8 else False

    def step(qq, kk, vv):
        return ulysses.exchange(qq, kk, vv, group, None, rows=rows, causal=cfg["causal"],
                                rope=spec, norm_q=norm, norm_k=norm, fp8=fp8_arg,
                                narrow=args.narrow)

    for _ in range(args.warmup):
        step(q, k, v)
    torch.cuda.synchronize()
    attention.check_status(device)
    ulysses.taken()
    if group is not None:
        dist.barrier()
    torch.cuda.synchronize()

    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # rank 0 samples its GPU's clocks (its line reports them); NVML queries from every rank's
    # process would take the driver beside the ranks' own launches
    sampler = clock_sampler(local_gpu_index(local)) if rank == 0 else NullSampler()
    with sampler:
        e0.record()
        for _ in range(args.steps):
            out = step(q, k, v)
        e1.record()
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    clock = ulysses.taken()
    attention.check_status(device)
    layout = ulysses.plan(rows, heads, hkv)
    calls = max(1, clock["calls"])
    attn_span = clock["attention_ms"] / calls
    stats = torch.tensor([ms, attn_span, clock["before_ms"] / calls, clock["after_ms"] / calls],
                         dtype=torch.float64, device=device)
    if group is not None:
        dist.all_reduce(stats, op=dist.ReduceOp.MAX)
    ms_max, span_max, before_max, after_max = stats.tolist()

    # ---- outside the timed region: the output checked, the attention alone, cuDNN, clocks
    extras: dict = {}
    if not args.no_extras and fp8:
        extras["parity"] = parity_check(q, k, v, out, rows, rank, group, cfg, spec, device,
                                        fp8=True)
        extras["first_stage"] = fp8_first_stage(q, k, v, layout, rank, args.fp8_law, spec,
                                                norm, max(3, args.steps // 2), device)
    if not args.no_extras and not fp8 and not args.narrow:
        extras["parity"] = parity_check(q, k, v, out, rows, rank, group, cfg, spec, device)
        alone = torch.tensor([attention_alone(cfg, layout, rank, max(3, args.steps // 4),
                                              device)], dtype=torch.float64, device=device)
        if group is not None:
            dist.all_reduce(alone, op=dist.ReduceOp.MAX)
        extras["attention_alone_ms"] = alone.item()
        if rank == 0:
            extras["cudnn"] = cudnn_attention(cfg, layout, rank, device)
    long_run = None
    if not args.no_extras and args.long_run_s > 0:
        # more steps until long_run_s has passed, each timed on the device: the median step and
        # the clocks of a timed region long enough to be steady
        if group is not None:
            dist.barrier()
        sampler_long = clock_sampler(local_gpu_index(local)) if rank == 0 else NullSampler()
        marks = []
        began = time.perf_counter()
        with sampler_long:
            while True:
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                step(q, k, v)
                b.record()
                marks.append((a, b))
                if len(marks) % 8 == 0:
                    torch.cuda.synchronize()
                    go = torch.tensor([time.perf_counter() - began < args.long_run_s],
                                      dtype=torch.int32, device=device)
                    if group is not None:  # every rank runs the same number of steps
                        dist.all_reduce(go, op=dist.ReduceOp.MIN)
                    if not go.item():
                        break
            torch.cuda.synchronize()
        per = torch.tensor([statistics.median(a.elapsed_time(b) for a, b in marks)],
                           dtype=torch.float64, device=device)
        if group is not None:
            dist.all_reduce(per, op=dist.ReduceOp.MAX)
        attention.check_status(device)
        ulysses.taken()
        long_run = {"steps": len(marks), "seconds": round(time.perf_counter() - began, 3),
                    "median_step_ms": round(per.item(), 4), "clocks": sampler_long.summary()}

    transport = ulysses.transport_of(group, device)
    flag_mode = None
    if transport == "peer":
        from cozy_runtime_b200 import peer

        flag_mode = peer.layer_group_for(group, device).flag_mode()
    links = None
    if group is not None and ulysses.links_of(group) is not None:
        links = ulysses.links_of(group).summary()  # the formation's per-pair probe
    crossing = None
    # the crossing of the bf16 layer (the FP8 and int8 wires store into the peers in-kernel)
    if transport == "peer" and group is not None and not fp8 and not args.narrow:
        # the latest call's crossing on each rank: its copy-engine copies to the other ranks and
        # their flag writes, timed on the side stream (bytes / time = the NVLink rate reached)
        torch.cuda.synchronize()
        got = peer.layer_group_for(group, device).crossing() or (0.0, 0)
        each = torch.tensor([got[0], float(got[1])], dtype=torch.float64, device=device)
        every = [torch.empty_like(each) for _ in range(world)]
        dist.all_gather(every, each)
        ms_each = [t[0].item() for t in every]
        bytes_each = [int(t[1].item()) for t in every]
        crossing = {
            "ms_max": round(max(ms_each), 4),
            "bytes_per_rank": bytes_each[0],
            "gbs_per_rank_min": round(min(b / (m * 1e-3) / 1e9 for b, m in
                                          zip(bytes_each, ms_each, strict=True) if m > 0), 1)
            if all(m > 0 for m in ms_each) else None,
            "how": "cudaMemcpyAsync peer copies on a side stream, beside the attention",
        }

    # ---- end to end through the public call, host buffers in and out every step
    e2e_ms = h2d = d2h = None
    if not args.no_e2e:
        # Every step copies its own inputs in from pinned host memory and its output back out, inside
        # the timed region; the copies run on their own streams, double-buffered, so step i+1's
        # inputs cross PCIe while step i computes and step i's output crosses while i+1 computes.
        hq = [t.cpu().pin_memory() for t in (q, k, v)]
        slots = [[torch.empty_like(t) for t in (q, k, v)] for _ in range(2)]
        host_outs = [torch.empty((batch, mine, heads, dim), dtype=torch.bfloat16).pin_memory()
                     for _ in range(2)]
        compute = torch.cuda.current_stream(device)
        h2d_stream, d2h_stream = torch.cuda.Stream(device), torch.cuda.Stream(device)
        loaded = [torch.cuda.Event() for _ in range(2)]
        freed = [torch.cuda.Event() for _ in range(2)]

        def issue_h2d(i):
            s = i % 2
            h2d_stream.wait_event(freed[s])  # the slot's previous step has read it
            with torch.cuda.stream(h2d_stream):
                for src, dst in zip(hq, slots[s], strict=True):
                    dst.copy_(src, non_blocking=True)
            loaded[s].record(h2d_stream)

        def run_step(i):
            s = i % 2
            compute.wait_event(loaded[s])
            result = step(*slots[s])
            freed[s].record(compute)
            d2h_stream.wait_event(freed[s])
            with torch.cuda.stream(d2h_stream):
                host_outs[s].copy_(result, non_blocking=True)
            result.record_stream(d2h_stream)

        def e2e_run(n):
            for ev in freed:
                ev.record(compute)
            h2d_stream.wait_stream(compute)
            d2h_stream.wait_stream(compute)
            issue_h2d(0)
            for i in range(n):
                if i + 1 < n:
                    issue_h2d(i + 1)
                run_step(i)
            compute.wait_stream(d2h_stream)

        e2e_run(2)
        torch.cuda.synchronize()
        if group is not None:
            dist.barrier()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e2e_steps = max(3, args.steps // 2)
        f0.record(compute)
        e2e_run(e2e_steps)
        f1.record(compute)
        torch.cuda.synchronize()
        e2e_ms = torch.tensor([f0.elapsed_time(f1) / e2e_steps], dtype=torch.float64, device=device)
        if group is not None:
            dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
        h2d = sum(t.numel() * t.element_size() for t in hq)
        d2h = host_outs[0].numel() * host_outs[0].element_size()

    flops = layer_flops(cfg)
    if rank == 0:
        burst, held, peak_src = peaks(fp8)
        sustained = ms_max / 1e3 >= SUSTAINED_STEP_S
        peak = held if sustained else burst
        my_flops = layer_flops(cfg, heads=layout.q_n[rank])
        alone_ms = extras.get("attention_alone_ms")
        # the dominant kernel's rate: alone (every operand resident) where measured, else its
        # span inside the layer (which includes waiting for rows still crossing)
        kernel_ms = alone_ms if alone_ms else span_max
        ach = my_flops / (kernel_ms * 1e-3) / 1e12 if kernel_ms else 0.0
        # my kernels a step: first stage + attention, then per transport the land (NCCL) or
        # the output flags' signal and wait kernels (peer: a copy-engine crossing is copies and
        # stream writes; an SM crossing adds the arrival flags' signal kernel, the gate a wait
        # kernel); FP8: statistics, e4m3 first stage and attention, over NVLink with the
        # arrival and output flags' signal and wait kernels
        kernels = 1 + (1 if (cfg["rope"] or cfg["norm"] or world > 1) else 0)
        if world > 1:
            kernels += {"peer": 2, "nccl": 1}.get(transport, 0)
            if transport == "peer" and not fp8 and not args.narrow:
                kernels += int(ulysses.layer_cross(world) == "sm") + int(ulysses.layer_gate(world))
        if fp8:
            kernels = 3 + ({"peer": 4, "nccl": 1}.get(transport, 0) if world > 1 else 0)
        if args.narrow:  # key sums, shift, pack, 3 widens, attention, return pack, land widen
            kernels = 9 + (2 if cfg["rope"] or cfg["norm"] else 0) + (
                4 if world > 1 and transport == "peer" else 0)
        profile = ROOT / "profiles" / f"attention_fwd_{args.config}_traffic.json"
        traffic = None
        if profile.exists():
            traffic = json.loads(profile.read_text()).get("dram_bytes_per_launch")
        exposed = ms_max - (alone_ms if alone_ms else span_max)
        line = {
            "metric": METRIC,
            "value": round(flops / (ms_max * 1e-3) / 1e12, 2),
            "unit": "TFLOP/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_max, 4),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "e4m3" if fp8 else "bf16",
            "data": "synthetic",
            "config": {
                "workload": cfg["workload"],
                "name": args.config,
                "batch": batch,
                "seq_len": seq,
                "heads": heads,
                "heads_kv": hkv,
                "head_dim": dim,
                "causal": cfg["causal"],
                "parallelism": f"ulysses{world}",
                "rows_per_rank": rows,
                "wire": "int8 (narrow)" if args.narrow else ("e4m3" if fp8 else "bf16"),
                **({"fp8_law": args.fp8_law} if fp8 else {}),
                "l2": "inputs larger than L2 (no flush)",
            },
            "transport": transport,
            "flag_mode": flag_mode,
            "layer_gate": ulysses.layer_gate(world) if transport == "peer" else None,
            "layer_cross": ulysses.layer_cross(world) if transport == "peer" else None,
            "crossing": crossing,
            "links": links,
            "layer": {
                "attention_span_ms": round(span_max, 4),
                "attention_alone_ms": None if alone_ms is None else round(alone_ms, 4),
                # exposed = layer - the attention alone: the crossing, first stage, flags and
                # copy-out that did not hide under the attention (max over ranks of each)
                "exposed_ms": round(exposed, 4),
                "exposed_frac": round(exposed / ms_max, 4) if ms_max else None,
                "before_attention_ms": round(before_max, 4),
                "after_attention_ms": round(after_max, 4),
            },
            "parity": extras.get("parity"),
            "first_stage": extras.get("first_stage"),
            "clocks": sampler.summary(),
            "long_run": long_run,
            "e2e": None if e2e_ms is None else {
                "value": round(flops / (e2e_ms.item() * 1e-3) / 1e12, 2),
                "unit": "TFLOP/s",
                "ms_per_step": round(e2e_ms.item(), 4),
                "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h,
                "call": "cozy_runtime_b200.ulysses.exchange(q, k, v, group, None, rope=...)",
                "pipelining": "H2D of step i+1 and D2H of step i on their own streams beside "
                "step i's compute (double-buffered inputs); every step's copies inside the "
                "timed region",
            },
            "gpu_launches": kernels * args.steps,
            "roofline": {
                "bound": "tensor",
                "kernel": f"attention_fwd_kernel<128, {'true' if fp8 else 'false'}>",
                "achieved": round(ach, 2),
                "peak": peak,
                "unit": "TFLOP/s",
                "frac": round(ach / peak, 4) if peak else None,
                "peak_source": peak_src + (" sustained (steps of 1 s or more)" if sustained
                                           else " burst"),
                "frac_of_sustained": round(ach / held, 4) if held else None,
                "measured_on": "the attention alone, operands resident" if alone_ms
                else "the attention's span inside the layer",
                "traffic": traffic,
            },
            "cudnn": extras.get("cudnn"),
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(cfg)
        print(json.dumps(line), flush=True)
    if group is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
