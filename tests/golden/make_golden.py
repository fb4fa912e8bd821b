"""Generate the golden vectors under tests/golden/ by running the REFERENCE's own code.

Test infrastructure only: this script imports cozy-runtime from a local checkout of the
reference named by `$COZY_REFERENCE_SRC` (the checkout's `src` directory; required) and is run
by hand in a container that has it. Nothing else in this repository imports it; the GPU box never runs it.

What it records, each as an `.npz` in this directory:

* ``ulysses_*.npz``: the reference's Ulysses exchange
  (`src/cozy_runtime/internal/parallel/ulysses.py:607` `exchange`) run over a gloo process group
  of W CPU processes, with `compute` = the reference's local kernel
  (`src/cozy_runtime/internal/attention_upstream.py:109` `sdpa`). Inputs are split along the
  sequence with `torch.tensor_split` (Diffusers' `ulysses_anything` split,
  `src/cozy_runtime/internal/parallel/cp.py:166-174`), the rank outputs are concatenated back in
  rank order. The causal-GQA case replicates K/V heads to the query heads first and passes
  `is_causal=True` to `sdpa`, as the exchange itself is mask-agnostic.
* ``rope_*.npz``: the reference's own eager RMSNorm+RoPE law, the checker inside
  `src/cozy_runtime/internal/bench/kernels.py:819` `_fused_rope`, executed with the Triton
  launch replaced by a recorder, so the recorded `want` is the reference code's output.
* ``fp8_quantise.npz``: `src/cozy_runtime/internal/attention_fp8.py:162` `quantise_eager`.
* ``fp8_head.npz``: the reference's FP8 row's quantisation, `attention_upstream.py:276`
  `_hadamard` of Q and K, then `quantise_eager` of the rotated Q, K and of V.
* ``turn_*.npz``: the int8 wire's law, `src/cozy_runtime/internal/parallel/turn.py:60`
  `law` (with and without a shift, which is `turned` of a mean as `_Shift` makes it) and `:73`
  `law_back`, on bf16 rows.
* ``narrow_*.npz``: the reference's exchange with `narrow=True` (Q, K less its turned mean, V
  and the output crossing as int8), bf16 inputs and `sdpa` in bf16, over gloo as above.

Run:  COZY_REFERENCE_SRC=<checkout>/src python tests/golden/make_golden.py [ulysses] [rope] [fp8] [turn] [narrow]  (default: all)
Third-party pins the reference declares but this container lacks (`tensorfs` 0.27.0,
`diffusers` 0.40.0) are replaced by import stubs: neither is on the computed path.
"""

from __future__ import annotations

import importlib.abc
import importlib.machinery
import os
import sys
import tempfile
from pathlib import Path
from unittest.mock import MagicMock

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REFERENCE_SRC = os.environ.get("COZY_REFERENCE_SRC", "")


class _Stub(importlib.abc.MetaPathFinder, importlib.abc.Loader):
    """Stub packages the reference imports but never computes with on this path."""

    roots = ("tensorfs", "diffusers")

    def find_spec(self, name, path, target=None):  # noqa: D102
        if name.split(".")[0] in self.roots:
            return importlib.machinery.ModuleSpec(name, self, is_package=True)
        return None

    def create_module(self, spec):  # noqa: D102
        module = MagicMock(name=spec.name)
        module.__path__ = []
        module.__spec__ = spec
        return module

    def exec_module(self, module):  # noqa: D102
        pass


def import_reference() -> None:
    if any(isinstance(f, _Stub) for f in sys.meta_path):
        return
    if not REFERENCE_SRC or not Path(REFERENCE_SRC, "cozy_runtime").is_dir():
        raise SystemExit("set COZY_REFERENCE_SRC to the reference checkout's src directory")
    sys.meta_path.insert(0, _Stub())
    meta = tempfile.mkdtemp(prefix="cozy-dist-")
    info = Path(meta, "cozy_runtime-0.0.0.dist-info")
    info.mkdir()
    (info / "METADATA").write_text("Metadata-Version: 2.1\nName: cozy-runtime\nVersion: 0.0.0\n")
    sys.path[:0] = [meta, REFERENCE_SRC]


def to_np(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)
    return t.contiguous().numpy()


# (name, world, batch, seq, heads_q, heads_kv, dim, compute dtype, causal). Inputs are drawn
# as bf16 values (the GPU path's input type) and the reference computes in `dtype` on them.
ULYSSES_CASES = [
    ("w1", 1, 1, 64, 4, 4, 64, torch.float32, False),
    ("w2_batch2", 2, 2, 45, 4, 4, 64, torch.float32, False),
    ("w3_padheads", 3, 1, 40, 5, 5, 128, torch.float32, False),
    ("w4_padheads", 4, 1, 50, 6, 6, 64, torch.float32, False),
    ("w4_bf16_compute", 4, 1, 50, 6, 6, 64, torch.bfloat16, False),
    ("w7_uneven", 7, 1, 50, 7, 7, 64, torch.float32, False),
    ("w2_causal_gqa", 2, 1, 33, 4, 2, 128, torch.float32, True),
    ("w7_causal_gqa_idle_ranks", 7, 1, 60, 8, 2, 64, torch.float32, True),
    ("w8", 8, 1, 37, 8, 8, 64, torch.float32, False),
]
SEED = 20261017  # the reference's attention self-check seed (internal/attention.py cases)


def _inputs(batch, seq, hq, hkv, dim, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(batch, seq, hq, dim, generator=g).to(torch.bfloat16).to(dtype)
    k = torch.randn(batch, seq, hkv, dim, generator=g).to(torch.bfloat16).to(dtype)
    v = torch.randn(batch, seq, hkv, dim, generator=g).to(torch.bfloat16).to(dtype)
    return q, k, v


def _rank(rank, world, port, case, outdir, narrow=False):
    import torch.distributed as dist

    import_reference()
    from cozy_runtime.internal import attention_upstream
    from cozy_runtime.internal.parallel import ulysses

    name, _, batch, seq, hq, hkv, dim, dtype, causal = case
    dist.init_process_group(
        "gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world
    )
    torch.set_num_threads(1)
    q, k, v = _inputs(batch, seq, hq, hkv, dim, dtype, SEED)
    if hkv != hq:  # the exchange serves equal heads: K/V replicated to the query heads
        k = k.repeat_interleave(hq // hkv, dim=2)
        v = v.repeat_interleave(hq // hkv, dim=2)
    parts = [torch.tensor_split(t, world, dim=1)[rank].contiguous() for t in (q, k, v)]
    out = ulysses.exchange(
        *parts,
        dist.group.WORLD,
        lambda a, b, c: attention_upstream.sdpa(a, b, c, is_causal=causal),
        site="golden",
        narrow=narrow,
    )
    torch.save(out, os.path.join(outdir, f"{name}.{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


def ulysses_goldens() -> None:
    import torch.multiprocessing as mp

    for index, case in enumerate(ULYSSES_CASES):
        name, world, batch, seq, hq, hkv, dim, dtype, causal = case
        with tempfile.TemporaryDirectory() as tmp:
            mp.spawn(_rank, args=(world, 29600 + index, case, tmp), nprocs=world, join=True)
            outs = [torch.load(os.path.join(tmp, f"{name}.{r}.pt")) for r in range(world)]
        out = torch.cat(outs, dim=1)
        q, k, v = _inputs(batch, seq, hq, hkv, dim, dtype, SEED)
        rows = [int(o.shape[1]) for o in outs]
        q, k, v = (t.to(torch.bfloat16) for t in (q, k, v))  # exact: drawn as bf16
        np.savez_compressed(
            HERE / f"ulysses_{name}.npz",
            q=to_np(q), k=to_np(k), v=to_np(v), out=to_np(out.float()), heads_kv=hkv,
            world=world, causal=int(causal), rows=np.array(rows),
            dtype=str(dtype).replace("torch.", ""),
        )
        print(f"ulysses_{name}: rows {rows} out {tuple(out.shape)} {out.dtype}")


# (name, HEADS, HEAD_DIM, ROTARY, INTERLEAVED, WEIGHT, OFFSET, ROUND, X32)
ROPE_CASES = [
    ("interleaved_full", 2, 64, 64, 1, 0, 0.0, 1, 0),
    ("split_half_full", 2, 64, 64, 0, 0, 0.0, 1, 0),
    ("interleaved_partial_weight", 2, 128, 96, 1, 1, 0.0, 1, 0),
    ("split_half_partial_weight_offset", 2, 128, 64, 0, 1, 1.0, 1, 0),
    ("interleaved_full_d128", 2, 128, 128, 1, 0, 0.0, 1, 0),
]


def rope_goldens() -> None:
    import_reference()
    from cozy_runtime.internal.bench import kernels as bench_kernels

    for name, heads, dim, rotary, inter, weight, offset, rnd, x32 in ROPE_CASES:
        entry = MagicMock()
        entry.key = name
        entry.constexprs = {
            "HEADS": heads, "HEAD_DIM": dim, "ROTARY": rotary, "INTERLEAVED": inter,
            "WEIGHT": weight, "OFFSET": offset, "ROUND": rnd, "X32": x32,
        }
        seen: dict[str, object] = {}

        def recorder(launch, entry_, x, w, eps, tables, out_type):
            seen.update(x=x.clone(), weight=w, eps=eps, tables=tables)
            return torch.zeros(x.shape, dtype=out_type)

        def error(torch_, got, want):
            seen["want"] = want.clone()
            return 0.0

        fused, verify = bench_kernels.fused, bench_kernels.verify
        saved = fused.head_norm_rope, verify.error
        fused.head_norm_rope, verify.error = recorder, error
        try:
            g = torch.Generator().manual_seed(8)
            bench_kernels._fused_rope(None, entry, torch.device("cpu"), g, {})
        finally:
            fused.head_norm_rope, verify.error = saved
        cos, sin, stride_token, stride_channel = seen["tables"]
        w = seen["weight"]
        np.savez_compressed(
            HERE / f"rope_{name}.npz",
            x=to_np(seen["x"]),
            weight=to_np(w.float()) if w is not None else np.zeros(0, np.float32),
            cos=cos.contiguous().numpy(), sin=sin.contiguous().numpy(),
            stride_token=stride_token, stride_channel=stride_channel,
            eps=seen["eps"], want=seen["want"].numpy(),
            rotary=rotary, interleaved=inter, has_weight=weight, offset=offset,
        )
        print(f"rope_{name}: x {tuple(seen['x'].shape)} strides ({stride_token},{stride_channel})")


def fp8_golden() -> None:
    import_reference()
    from cozy_runtime.internal import attention_fp8

    g = torch.Generator().manual_seed(SEED)
    x = torch.randn(2, 70, 3, 64, generator=g).to(torch.bfloat16)
    x[1, :, 2] = 0  # an all-zero head takes the scale floor
    x[0, 5, 1, 7] = 40.0
    codes, descale = attention_fp8.quantise_eager(x)
    np.savez_compressed(
        HERE / "fp8_quantise.npz",
        x=to_np(x), codes=codes.view(torch.uint8).numpy(), descale=descale.numpy(),
    )
    print("fp8_quantise:", tuple(codes.shape), tuple(descale.shape))

    # The reference's own FP8 row on B200 (`fa4_fp8`): Q and K rotated by `_hadamard` (a bf16
    # matrix product), then Q, K and V quantised per (batch, head) by `quantise` (on the CPU its
    # eager law). Recorded: the rotated Q and K, and every code and descale.
    from cozy_runtime.internal import attention_upstream

    g = torch.Generator().manual_seed(SEED + 1)
    q, k, v = (torch.randn(2, 200, 3, 128, generator=g) for _ in range(3))
    k = torch.where(torch.rand(k.shape, generator=g) < 0.01, k * 8, k)
    q, k, v = (t.to(torch.bfloat16) for t in (q, k, v))
    rq, rk = attention_upstream._hadamard(q), attention_upstream._hadamard(k)
    out = {"q": to_np(q), "k": to_np(k), "v": to_np(v), "rq": to_np(rq), "rk": to_np(rk)}
    for name, t in (("q", rq), ("k", rk), ("v", v)):
        codes, descale = attention_fp8.quantise_eager(t)
        out[f"{name}_codes"] = codes.view(torch.uint8).numpy()
        out[f"{name}_descale"] = descale.numpy()
    np.savez_compressed(HERE / "fp8_head.npz", **out)
    print("fp8_head:", tuple(q.shape))


# (name, world, batch, seq, heads_q, heads_kv, dim, causal): bf16 inputs and compute
NARROW_CASES = [
    ("w1", 1, 1, 48, 2, 2, 64, False),
    ("w2_batch2", 2, 2, 37, 4, 4, 128, False),
    ("w3_padheads", 3, 1, 40, 4, 4, 64, False),
    ("w2_causal_gqa", 2, 1, 33, 4, 2, 128, True),
]


def narrow_goldens() -> None:
    import torch.multiprocessing as mp

    for index, (name, world, batch, seq, hq, hkv, dim, causal) in enumerate(NARROW_CASES):
        case = (name, world, batch, seq, hq, hkv, dim, torch.bfloat16, causal)
        with tempfile.TemporaryDirectory() as tmp:
            mp.spawn(_rank, args=(world, 29700 + index, case, tmp, True), nprocs=world, join=True)
            outs = [torch.load(os.path.join(tmp, f"{name}.{r}.pt")) for r in range(world)]
        out = torch.cat(outs, dim=1)
        q, k, v = _inputs(batch, seq, hq, hkv, dim, torch.bfloat16, SEED)
        rows = [int(o.shape[1]) for o in outs]
        np.savez_compressed(
            HERE / f"narrow_{name}.npz",
            q=to_np(q), k=to_np(k), v=to_np(v), out=to_np(out), heads_kv=hkv, world=world,
            causal=int(causal), rows=np.array(rows),
        )
        print(f"narrow_{name}: rows {rows} out {tuple(out.shape)} {out.dtype}")


def turn_goldens() -> None:
    import_reference()
    from cozy_runtime.internal.parallel import turn

    for dim in (64, 128):
        g = torch.Generator().manual_seed(SEED + dim)
        x = torch.randn(2, 40, 3, dim, generator=g).to(torch.bfloat16)
        x[0, 3, 1] = 0  # an all-zero row takes the scale floor
        x[1, 7, 2, 5] = 60.0  # an outlier
        key = (torch.randn(2, 40, 3, dim, generator=g) + 0.7).to(torch.bfloat16)
        summed = key.sum(1, dtype=torch.float32)
        shift = turn.turned(summed / key.shape[1])  # as `_Shift` makes it
        codes, scale = turn.law(x)
        kcodes, kscale = turn.law(key, shift[:, None])
        np.savez_compressed(
            HERE / f"turn_d{dim}.npz",
            x=to_np(x), codes=codes.numpy(), scale=to_np(scale), back=to_np(turn.law_back(codes, scale)),
            key=to_np(key), shift=shift.numpy(), kcodes=kcodes.numpy(), kscale=to_np(kscale),
            kback=to_np(turn.law_back(kcodes, kscale)),
        )
        print(f"turn_d{dim}: codes {tuple(codes.shape)} scale {tuple(scale.shape)}")


if __name__ == "__main__":
    import sys as _sys

    parts = set(_sys.argv[1:]) or {"ulysses", "rope", "fp8", "turn", "narrow"}
    if "ulysses" in parts:
        ulysses_goldens()
    if "rope" in parts:
        rope_goldens()
    if "fp8" in parts:
        fp8_golden()
    if "turn" in parts:
        turn_goldens()
    if "narrow" in parts:
        narrow_goldens()
