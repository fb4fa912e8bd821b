"""Host logic without a GPU: head ownership, row splits, the store meeting over gloo ranks, and the
C ABI library's exports (no compute calls)."""

import ctypes
import os
import re
from pathlib import Path

import pytest
import torch

import oracle

ROOT = Path(__file__).resolve().parent.parent


def test_plan_matches_oracle_head_ownership():
    from cozy_runtime_b200 import ulysses

    for heads in (5, 7, 8, 24, 32, 40):
        for world in (1, 2, 3, 4, 7, 8):
            layout = ulysses.plan([10] * world, heads, heads)
            for r in range(world):
                owned = oracle.owned_heads(heads, world, r)
                assert layout.q_lo[r] == (owned.start if len(owned) else layout.q_lo[r])
                assert layout.q_n[r] == len(owned)


def test_plan_gqa_kv_heads_cover_query_heads():
    from cozy_runtime_b200 import ulysses

    for hq, hkv in ((32, 8), (8, 2), (24, 24), (40, 8)):
        for world in (1, 2, 4, 7, 8):
            lay = ulysses.plan([3] * world, hq, hkv)
            for r in range(world):
                for h in range(lay.q_lo[r], lay.q_lo[r] + lay.q_n[r]):
                    kvh = h // lay.group
                    assert lay.kv_lo[r] <= kvh < lay.kv_lo[r] + lay.kv_n[r]


def test_c5_degree7_ownership():
    """Causal GQA prefill at degree 7: 32 query heads pad to 35, ranks own 5,5,5,5,5,5,2."""
    from cozy_runtime_b200 import ulysses

    rows = ulysses.tensor_split_rows(131071, 7)
    assert rows == [18725, 18725, 18725, 18724, 18724, 18724, 18724]
    lay = ulysses.plan(rows, 32, 8)
    assert lay.q_n == (5, 5, 5, 5, 5, 5, 2)
    assert lay.kv_n == (2, 2, 2, 2, 2, 2, 1)


def test_tensor_split_rows():
    from cozy_runtime_b200 import ulysses

    for total in (7, 4608, 33272, 131071):
        for world in (1, 2, 4, 7, 8):
            want = [t.shape[0] for t in torch.tensor_split(torch.empty(total), world)]
            assert ulysses.tensor_split_rows(total, world) == want


def _meeting_rank(rank, world, port, results):
    import torch.distributed as dist

    from cozy_runtime_b200 import ulysses

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    meet = ulysses._meeting(dist.group.WORLD)
    first = meet.gather({"rows": 10 + rank, "site": "a"})
    second = meet.gather({"rows": 20 + rank, "site": "a"})
    diverged = ""
    try:
        meet.gather({"rows": 1, "site": f"site{rank}"})
    except RuntimeError as exc:
        diverged = str(exc)
    results[rank] = ([r["rows"] for r in first], [r["rows"] for r in second], diverged)
    dist.barrier()
    dist.destroy_process_group()


def test_store_meeting_gloo_world2():
    """Two gloo ranks agree on each other's rows per call and both see a divergence."""
    import torch.multiprocessing as mp

    manager = mp.Manager()
    results = manager.dict()
    mp.spawn(_meeting_rank, args=(2, 29731, results), nprocs=2, join=True)
    for rank in range(2):
        first, second, diverged = results[rank]
        assert first == [10, 11] and second == [20, 21]
        assert "is not one call" in diverged


def _header_symbols() -> set[str]:
    text = (ROOT / "include" / "cozy_ulysses.h").read_text()
    return set(re.findall(r"COZY_API\s+[\w\s\*]+?\b(cozy_\w+)\s*\(", text))


def test_library_exports_header_symbols():
    from cozy_runtime_b200 import _lib

    lib = ctypes.CDLL(str(_lib.LIBRARY))
    declared = _header_symbols()
    assert declared == set(_lib.SIGNATURES), "the ctypes binding covers the header"
    for name in declared:
        assert hasattr(lib, name), name
    assert lib.cozy_abi_version() == 104


def test_error_name_without_gpu():
    from cozy_runtime_b200 import _lib

    assert _lib.error_name(801) == "cudaErrorNotSupported"
    assert _lib.error_name(0) == "cudaSuccess"


def test_product_path_fails_loudly_without_library(monkeypatch, tmp_path):
    from cozy_runtime_b200 import _lib

    monkeypatch.setattr(_lib, "_LIB", None)
    monkeypatch.setattr(_lib, "LIBRARY", tmp_path / "missing.so")
    with pytest.raises(RuntimeError, match="not built"):
        _lib.load()


def test_product_does_not_import_oracle():
    for path in (ROOT / "cozy_runtime_b200").rglob("*.py"):
        text = path.read_text()
        assert "import oracle" not in text and "from oracle" not in text, path


def test_exchange_refuses_cpu():
    """No CPU fallback: host tensors are refused, on the int8 wire too."""
    from cozy_runtime_b200 import ulysses

    x = torch.zeros(1, 4, 2, 64, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        ulysses.exchange(x, x, x, None, None, narrow=True)
    with pytest.raises(ValueError):
        ulysses.exchange(x, x, x, None, None)


def test_destination_order_is_a_permutation_at_every_step():
    """At every position of the first stage's destination lists the ranks target distinct
    peers, and each rank's list covers every peer once."""
    from cozy_runtime_b200 import ulysses

    for world in (1, 2, 3, 4, 7, 8):
        orders = [ulysses.destination_order(r, world) for r in range(world)]
        for r in range(world):
            assert sorted(orders[r]) == list(range(world)) and orders[r][0] == r
        for i in range(world):
            assert sorted(o[i] for o in orders) == list(range(world))


def test_narrow_block_sizes_cover_the_exchange():
    """The int8 wire's per-peer blocks add up to the whole exchange in both directions: what
    every rank sends for Q equals what the rank holding those heads receives, and the return
    blocks of every source fill each rank's output rows of every head."""
    from cozy_runtime_b200 import narrow, ulysses

    batch, dim = 2, 64
    for total, world, heads, hkv in ((100, 3, 5, 5), (37, 8, 16, 4), (50, 4, 6, 2)):
        rows = ulysses.tensor_split_rows(total, world)
        lay = ulysses.plan(rows, heads, hkv)
        steps = []
        for r in range(world):
            q = torch.empty(batch, rows[r], heads, dim, dtype=torch.bfloat16)
            kv = torch.empty(batch, rows[r], hkv, dim, dtype=torch.bfloat16)
            steps.append(narrow.NarrowStep(q, kv, kv, lay, r))
        for p in range(world):
            got_q = sum(st.first_block(p, "q") for st in steps)
            assert got_q == total * batch * lay.q_n[p] * dim
            got_kv = sum(st.first_block(p, "kv") for st in steps)
            assert got_kv == total * batch * lay.kv_n[p] * dim
        for r, st in enumerate(steps):
            # a source's return block to owner r is that owner's landing block from the source
            for s in range(world):
                assert steps[s].return_block(r) == st.landing_block(s)
            assert sum(st.landing_block(s) for s in range(world)) == rows[r] * batch * heads * dim


def test_scale_pointer_of_a_block():
    from cozy_runtime_b200 import narrow

    codes, scales = 1 << 20, 1 << 30
    assert narrow.scale_ptr(codes, scales, 0, 128) == (codes, scales)
    # 3 rows of 128 codes in: 3 bf16 scales in
    assert narrow.scale_ptr(codes, scales, 3 * 128, 128) == (codes + 384, scales + 6)


def _plan(batch, seq, heads, causal=False, sms=148, dim=128):
    from cozy_runtime_b200 import _lib

    whole, parts = ctypes.c_longlong(), ctypes.c_int()
    code = _lib.load().cozy_attention_split_plan_for(
        batch, seq, seq, heads, dim, int(causal), sms, ctypes.byref(whole), ctypes.byref(parts))
    assert code == 0
    return whole.value, parts.value


def test_split_plan_for_the_benchmark_shapes():
    """The attention's schedule on 148 SMs (host arithmetic, no GPU): C2 splits its last
    partial wave at degrees 4 and 8 (5.27 and 2.64 waves), not at 1 (21 waves: the SMs' drift
    absorbs it) nor at 2 (a predicted 3 %, under the 5 % bar); causal calls never split."""
    c2 = 33272
    assert _plan(1, c2, 24) == (3120, 1)
    assert _plan(1, c2, 12) == (1560, 1)
    assert _plan(1, c2, 6) == (740, 7)
    assert _plan(1, c2, 3) == (296, 3)
    assert _plan(1, 131071, 32, causal=True) == (16384, 1)
    whole, parts = _plan(2, 4608, 6)  # C3 at degree 4: one whole wave, the rest split
    assert whole == 148 and parts > 1
    whole, parts = _plan(1, 4000, 2)  # fewer tiles than SMs: all split
    assert whole == 0 and parts > 1
    assert _plan(1, 256 * 148, 1)[1] == 1  # exactly one wave


def test_split_plan_refuses_bad_arguments():
    from cozy_runtime_b200 import _lib

    whole, parts = ctypes.c_longlong(), ctypes.c_int()
    lib = _lib.load()
    assert lib.cozy_attention_split_plan_for(1, 100, 100, 2, 96, 0, 148, ctypes.byref(whole),
                                             ctypes.byref(parts)) != 0
    assert lib.cozy_attention_split_plan_for(1, 100, 100, 2, 128, 0, 0, ctypes.byref(whole),
                                             ctypes.byref(parts)) != 0


def test_backend_call_refusals_without_gpu():
    """The backend call's refusals, which come before any device work, as the reference's
    (attention_ulysses.py:246-262): log-sum-exp, masks under Ulysses, a kernel that is not
    head-local, ring attention."""
    from types import SimpleNamespace

    from cozy_runtime_b200 import attention_ulysses as au

    x = torch.zeros(1, 4, 2, 64, dtype=torch.bfloat16)
    call = au._dispatch("cozy_b200_test", au.COZY_B200)
    with pytest.raises(ValueError, match="log-sum-exp"):
        call(x, x, x, return_lse=True)
    config = SimpleNamespace(context_parallel_config=SimpleNamespace(ring_degree=1, group=None))
    with pytest.raises(ValueError, match="unmasked"):
        call(x, x, x, attn_mask=torch.zeros(4, 4, dtype=torch.bool), _parallel_config=config)
    # grouped-query heads under Ulysses need enable_gqa
    kv = torch.zeros(1, 4, 1, 64, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        call(x, kv, kv, _parallel_config=config)
    reducing = au.Local(forward=lambda *a, **k: None, impl=lambda *a: "", head_local=False)
    with pytest.raises(ValueError, match="head"):
        au._dispatch("reducing_test", reducing)(x, x, x, _parallel_config=config)
    ring = SimpleNamespace(context_parallel_config=SimpleNamespace(ring_degree=2))
    with pytest.raises(ValueError, match="ring"):
        au.group(ring)
    with pytest.raises(ValueError, match="not initialized"):
        au.group(SimpleNamespace(context_parallel_config=SimpleNamespace(ring_degree=1)))


def test_candidate_row_matches_the_kernel():
    from cozy_runtime_b200 import attention_ulysses as au

    row = au.CANDIDATE
    assert row.families == frozenset({"tcgen05"}) and row.dtypes == ("bfloat16",)
    assert row.head_dims == (64, 128) and row.causal and row.gqa and not row.masks
    assert row.local is au.COZY_B200 and row.local.head_local


def _crossing_rank(rank, world, port, outdir):
    import time
    from datetime import timedelta

    import torch.distributed as dist

    from cozy_runtime_b200 import ulysses

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=timedelta(seconds=5))
    group = dist.group.WORLD
    x = torch.arange(4 * world, dtype=torch.float32) + 100 * rank
    got = torch.empty_like(x)
    began = time.perf_counter()
    outcome = "returned"
    try:
        with ulysses._Crossing(group) as crossing:
            crossing.crossed = True
            dist.all_to_all_single(got, x, group=group)  # the first crossing
            if rank == 1:
                raise ValueError("compute failed after the crossing")
            back = torch.empty_like(x)
            dist.all_to_all_single(back, got, group=group)  # the return: rank 1 never comes
    except ValueError:
        outcome = "ValueError"
    except RuntimeError:
        outcome = "RuntimeError"
    elapsed = time.perf_counter() - began
    with open(os.path.join(outdir, f"{rank}.txt"), "w") as fh:
        fh.write(f"{outcome} {elapsed:.1f}")


def test_failure_after_crossing_ends_the_wait_of_peers():
    """A rank whose compute raises after the first crossing ends its group on the way out (the
    reference's abort_process_group after a crossing): the peer blocked in the return crossing
    raises within the group's timeout instead of waiting for it. Two gloo ranks on CPU."""
    import socket
    import tempfile

    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    with tempfile.TemporaryDirectory() as tmp:
        mp.spawn(_crossing_rank, args=(2, port, tmp), nprocs=2, join=True)
        outcomes = [open(os.path.join(tmp, f"{r}.txt")).read().split() for r in range(2)]
    assert outcomes[1][0] == "ValueError"
    assert outcomes[0][0] == "RuntimeError" and float(outcomes[0][1]) < 60


# ------------------------------------------------------------------------------ link probe
def test_links_route_from_pairs():
    """The route follows from the measured pairs alone (the reference's `Links.exchange`):
    every ordered pair direct -> the NVLink layer; one slow pair -> NCCL, and `why` names it."""
    from cozy_runtime_b200 import links

    fast = [[0, 750, 760], [740, 0, 755], [770, 745, 0]]
    found = links.decide(fast, [18, 18, 18])
    assert found.exchange == "peer" and found.all_direct and len(found.pairs) == 6
    assert found.summary()["min_gbs"] == 740.0
    slow = [row[:] for row in fast]
    slow[2][0] = 48.0  # a PCIe-class pair
    found = links.decide(slow, [18, 18, 0])
    assert found.exchange == "nccl" and not found.all_direct
    assert "2->0" in found.why()
    unmapped = links.decide(fast, peers=[[True, True, True], [True, True, False], [True] * 3])
    assert unmapped.exchange == "nccl" and not unmapped.all_peers


def test_links_nvml_count_with_a_fake_nvml():
    """NVML's active link count (read-only queries), against a stand-in NVML; -1 without one."""
    from cozy_runtime_b200 import links

    class FakeNvml:
        NVML_FEATURE_ENABLED = 1
        NVML_NVLINK_MAX_LINKS = 18

        def nvmlInit(self):
            pass

        def nvmlDeviceGetHandleByIndex(self, index):
            return index

        def nvmlDeviceGetNvLinkState(self, handle, link):
            if link >= 18:
                raise RuntimeError("no such link")
            return 1 if link < 18 - handle else 0

    assert links.nvlink_links(0, FakeNvml()) == 18
    assert links.nvlink_links(3, FakeNvml()) == 15

    class Broken:
        def nvmlInit(self):
            raise RuntimeError("driver not loaded")

    assert links.nvlink_links(0, Broken()) == -1


def _links_rank(rank, world, port, out):
    import torch.distributed as dist

    from cozy_runtime_b200 import links

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)

    class FakeLayer:  # the layer group's probe: rank 1 -> 0 is a slow pair
        def probe(self, dst, reps):
            gbs = 40.0 if (rank, dst) == (1, 0) else 700.0
            nbytes = 1 << 26
            return nbytes / (gbs * 1e9) * 1e3, nbytes

    found = links.measure(FakeLayer(), dist.group.WORLD, torch.device("cpu"))
    with open(os.path.join(out, f"{rank}.txt"), "w") as fh:
        fh.write(f"{found.exchange}|{found.why()}")
    dist.destroy_process_group()


def test_links_measure_over_gloo_ranks(tmp_path):
    """`links.measure` over two CPU ranks with a stand-in probe: both ranks gather the same rate
    matrix and take the same route (NCCL: the 1->0 pair is slow)."""
    import socket

    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.spawn(_links_rank, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    got = [open(tmp_path / f"{r}.txt").read() for r in range(2)]
    assert got[0] == got[1] and got[0].startswith("nccl|") and "1->0" in got[0]


# ------------------------------------------------------------------------ bench reference arm
def _bench(*args, env=None):
    import subprocess
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    return subprocess.run([sys.executable, os.path.join(root, "bench.py"), *args], cwd=root,
                          env={**os.environ, **(env or {})}, capture_output=True, text=True,
                          timeout=300)


def test_bench_reference_arm_line():
    """`bench.py --impl reference` prints one JSON line with the contract's keys: the reference
    arm's value, its cpu_baseline (kind, cores, sample) and an e2e with no device copies."""
    import json

    run = _bench("--impl", "reference", "--steps", "1", "--warmup", "0")
    assert run.returncode == 0, run.stderr[-2000:]
    line = json.loads(run.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["value"] > 0 and line["n_gpus"] == 1
    base = line["cpu_baseline"]
    assert base["kind"] in ("port", "reference") and base["cores"] >= 1 and base["sample"]
    assert base["value"] == line["value"]
    assert line["e2e"] == {"value": line["value"], "unit": line["unit"],
                           "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_bench_reference_arm_other_ranks_exit_quietly():
    """Under torchrun the reference arm runs on rank 0 alone; other ranks exit 0 and print
    nothing."""
    run = _bench("--impl", "reference", "--gpus", "2", "--steps", "1", "--warmup", "0",
                 env={"RANK": "1", "LOCAL_RANK": "1", "WORLD_SIZE": "2"})
    assert run.returncode == 0, run.stderr[-2000:]
    assert run.stdout.strip() == ""


# ------------------------------------------------------------------- context-parallel types
def test_group_mesh_serves_the_backend_its_group():
    """A parallel config built from `CpComms` and `GroupMesh` (the reference's cp.py:32-77)
    hands `attention_ulysses.group` its process group; the ring axis refuses."""
    from cozy_runtime_b200 import attention_ulysses, cp

    sentinel = object()
    mesh = cp.GroupMesh(cp.CpComms(pg=sentinel, rank=1, device="cpu"), size=4, local_rank=1)
    assert mesh.size() == 4 and mesh.get_local_rank() == 1
    assert mesh["ulysses"].get_group() is sentinel and mesh[("ulysses",)].get_group() is sentinel
    with pytest.raises(cp.ContextParallelUnavailable):
        mesh["ring"].get_group()
    with pytest.raises(KeyError):
        mesh["tensor"]

    class ContextParallelConfig:
        ring_degree = 1
        _ulysses_mesh = mesh

    class ParallelConfig:
        context_parallel_config = ContextParallelConfig()

    attention_ulysses.serve(None)
    assert attention_ulysses.group(ParallelConfig()) is sentinel
    ContextParallelConfig.ring_degree = 2
    with pytest.raises(ValueError):
        attention_ulysses.group(ParallelConfig())


def test_layer_crossing_policy(monkeypatch):
    """The NVLink layer crosses by SM stores from degree 4 and by copy engines below (the
    measured choice), unless `COZY_LAYER_CROSS` forces one; the gate is off unless forced."""
    from cozy_runtime_b200 import ulysses

    monkeypatch.delenv("COZY_LAYER_CROSS", raising=False)
    monkeypatch.delenv("COZY_LAYER_GATE", raising=False)
    assert [ulysses.layer_cross(w) for w in (2, 3, 4, 7, 8)] == ["ce", "ce", "sm", "sm", "sm"]
    assert not ulysses.layer_gate(8)
    monkeypatch.setenv("COZY_LAYER_CROSS", "ce")
    monkeypatch.setenv("COZY_LAYER_GATE", "1")
    assert ulysses.layer_cross(8) == "ce" and ulysses.layer_gate(2)
