"""CPU unit tests: selector tables, crossover detection, configuration,
reference-compatible exports and IPC handle serialisation (no GPU needed)."""

import json
import pickle

import pytest
import torch


def test_build_table_merges_and_covers_everything():
    from b200ar.parallel.selector import build_table

    rows = []
    for size, best in ((4096, "lamport"), (8192, "lamport"), (1 << 20, "twoshot"), (1 << 28, "nccl")):
        for v in ("lamport", "twoshot", "nccl"):
            rows.append({"bytes": size, "variant": v, "ctas": 8, "us": 1.0 if v == best else 5.0})
    table = build_table(rows)
    assert [e[1] for e in table] == ["lamport", "twoshot", "nccl"]
    assert table[0][0] == 8192 and table[1][0] == 1 << 20
    assert table[-1][0] >= 1 << 62  # the last entry covers every larger size


def test_crossover_bytes():
    from b200ar.parallel.selector import crossover_bytes

    rows = []
    for s, (ours, nccl) in {1: (1, 2), 2: (1, 2), 4: (3, 2), 8: (5, 2)}.items():
        rows += [{"bytes": s, "impl": "custom", "us": ours}, {"bytes": s, "impl": "nccl", "us": nccl}]
    assert crossover_bytes(rows) == 4
    rows = [{"bytes": 1, "impl": "custom", "us": 1}, {"bytes": 1, "impl": "nccl", "us": 2}]
    assert crossover_bytes(rows) is None


def test_load_table_picks_nearest_world(tmp_path):
    from b200ar.parallel.selector import FALLBACK, load_table, save_tables

    p = tmp_path / "t.json"
    save_tables(str(p), {2: [(100, "lamport", 1)], 8: [(200, "twoshot", 4)]})
    assert load_table(2, str(p)) == [(100, "lamport", 1)]
    assert load_table(6, str(p)) == [(200, "twoshot", 4)]
    assert load_table(3, str(p)) == [(100, "lamport", 1)]
    assert load_table(4, str(p)) == [(200, "twoshot", 4)]  # log-scale tie -> larger world
    assert load_table(4, str(tmp_path / "missing.json")) == FALLBACK
    data = json.loads(p.read_text())
    assert set(data["tables"]) == {"2", "8"}


def test_packaged_table_is_valid():
    from b200ar.parallel.selector import VARIANTS, load_table

    for w in (2, 4, 8):
        table = load_table(w)
        assert table and all(v in VARIANTS for _, v, _ in table)
        sizes = [b for b, _, _ in table]
        assert sizes == sorted(sizes)


def test_variant_ids_roundtrip():
    from b200ar.parallel.selector import VARIANT_NAMES, VARIANTS, variant_id

    for name, vid in VARIANTS.items():
        assert variant_id(name) == vid and VARIANT_NAMES[vid] == name
    with pytest.raises(ValueError):
        variant_id("nope")


def test_config_env_overrides(monkeypatch):
    from b200ar.config import default_config

    monkeypatch.setenv("B200AR_MAX_SIZE", "1234")
    monkeypatch.setenv("B200AR_NVLS", "1")
    cfg = default_config({"timeout_ms": 7})
    assert cfg.max_size == 1234 and cfg.enable_nvls and cfg.timeout_ms == 7


def test_compat_exports_match_reference_api():
    import b200ar.compat as c

    names = ["init_custom_ar", "all_reduce", "dispose", "meta_size", "register_buffer", "register_pcie_buffers",
             "get_graph_buffer_ipc_meta", "register_graph_buffers"]
    assert sorted(c.__all__) == sorted(names)
    for n in names:
        assert callable(getattr(c, n))
    assert c.meta_size() > 0 and c.meta_size() % 256 == 0


def test_ipc_handle_pickles():
    from b200ar.ipc import HANDLE_BYTES, cudaIpcMemHandle_t

    raw = bytes(range(HANDLE_BYTES))
    h = cudaIpcMemHandle_t.from_bytes(raw)
    h2 = pickle.loads(pickle.dumps(h))
    assert h2.to_bytes() == raw
    with pytest.raises(ValueError):
        cudaIpcMemHandle_t.from_bytes(b"short")


def test_slot_bytes_formulas():
    from b200ar import _C
    from b200ar.parallel.selector import VARIANTS

    assert _C.variant_slot_bytes(VARIANTS["oneshot_push"], 1024, 8) == 8192
    assert _C.variant_slot_bytes(VARIANTS["oneshot_pull"], 1024, 8) == 1024
    # two-shot: (world + 1) parts of ceil(packets / world) packets
    assert _C.variant_slot_bytes(VARIANTS["twoshot"], 16 * 10, 4) == 5 * 3 * 16
    assert _C.lamport_bytes(1024, 8) == 3 * 8 * 1024
    assert _C.gemm_ar_slot_bytes(128, 256, 2) == 3 * 1 * 128 * 256 * 2


def test_allocator_settings_that_block_ipc(monkeypatch):
    from b200ar import ipc

    for var in ("PYTORCH_CUDA_ALLOC_CONF", "PYTORCH_ALLOC_CONF"):
        monkeypatch.delenv(var, raising=False)
    assert ipc.allocator_blocks_ipc() is None
    monkeypatch.setenv("PYTORCH_CUDA_ALLOC_CONF", "max_split_size_mb:128,expandable_segments:True")
    assert "expandable_segments" in ipc.allocator_blocks_ipc()
    monkeypatch.setenv("PYTORCH_CUDA_ALLOC_CONF", "expandable_segments:False")
    assert ipc.allocator_blocks_ipc() is None
    monkeypatch.setenv("PYTORCH_ALLOC_CONF", "backend:cudaMallocAsync")
    assert "cudaMallocAsync" in ipc.allocator_blocks_ipc()

    def failing_export(ptr):
        raise RuntimeError("CUDA error: invalid argument")

    monkeypatch.setattr(ipc._C, "ipc_get_handle", failing_export)
    with pytest.raises(RuntimeError, match="CudaIPC\\(\\).malloc"):
        ipc.export_handle(0x1000)
    monkeypatch.delenv("PYTORCH_ALLOC_CONF")
    with pytest.raises(RuntimeError, match="^CUDA error"):  # no setting to blame: the original error
        ipc.export_handle(0x1000)


def test_latency_stats_and_bandwidth():
    from b200ar.utils.timing import NVLINK_GBS, allreduce_bandwidth, latency_stats

    st = latency_stats([float(v) for v in range(1, 12)])  # 1..11 us
    assert st == {"p10": 2.0, "p50": 6.0, "p90": 10.0, "max": 11.0}
    bw = allreduce_bandwidth(1 << 30, 8, 1e6 * (1 << 30) / 700e9)  # 1 GiB in the time of 700 GB/s algbw
    assert bw["algbw_gbs"] == 700.0
    assert bw["busbw_gbs"] == round(700.0 * 14 / 8, 1)
    assert bw["busbw_frac_of_nvlink"] == round(700.0 * 14 / 8 / NVLINK_GBS, 3)
    assert allreduce_bandwidth(4096, 1, 1.0)["busbw_gbs"] == 0.0


def test_render_md_tables(tmp_path):
    import importlib.util
    import os

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    spec = importlib.util.spec_from_file_location("render_md", os.path.join(root, "bench", "render_md.py"))
    rm = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(rm)
    ours = {"impl": "b200ar", "n_gpus": 2, "metric": "m", "value": 1.0, "unit": "us",
            "sweep": [{"bytes": 4096, "variant": "lamport", "eager_p50_us": 10.0, "graph_p50_us": 8.0,
                       "eager_us": {"p10": 9.0, "p50": 10.0, "p90": 12.0, "max": 20.0},
                       "nccl_eager_p50_us": 20.0, "busbw_gbs": 0.4, "busbw_frac_of_nvlink": 0.001}],
            "crossover_bytes": {"eager": None}, "clocks": {"sm_mhz": 1965, "sm_max_mhz": 1965, "reasons": []}}
    ref = {"impl": "reference", "sweep": [{"bytes": 4096, "eager_p50_us": 30.0}]}
    md = rm.render(ours, ref)
    assert "| 4096 | lamport | 10.00 (9.00-12.00) | 8.00 | 20.00 | 2.00x | 0.4 | 0.00 | 30.00 | 3.00x |" in md
    assert "crossover" in md and "1965 of 1965" in md
    assert "unavailable" in rm.render({"impl": "reference", "unavailable": "odd world"})
    p = tmp_path / "r.json"
    p.write_text("NCCL version banner\n" + json.dumps(ours) + "\n")
    assert len(rm.load_lines(str(p))) == 1
    # Recorded TP8 lines render: a detailed one (per-size sweep) and a printed
    # one (compact rows only).
    for name in ("bench_line_tp8_detailed.json", "bench_line_tp8.json"):
        committed = rm.load_lines(os.path.join(root, "tests", "data", name))
        assert committed and "| 268435456 |" in rm.render(committed[-1], committed[-1]), name


def test_rank_data_arena_bookkeeping():
    from b200ar import _C

    rec = int(_C.RANK_DATA_BYTES)
    assert rec == 8 * 8  # one pointer per rank, kMaxRanks = 8
    base = 0x7F0000000000  # addresses only: the arena never dereferences them
    a = _C.RankDataArena(base, 10 * rec + rec // 2)
    assert (a.capacity, a.used, a.remaining) == (10, 0, 10)
    assert a.take(3) == base
    # Capture reserves records by position without taking them.
    assert a.peek(0) == base + 3 * rec and a.peek(2) == base + 5 * rec
    assert a.take(1) == base + 3 * rec
    assert a.fits(6) and not a.fits(7) and not a.fits(-1)
    with pytest.raises(RuntimeError, match="overflow: 7 record"):
        a.take(7)
    assert a.used == 4  # a failed take leaves the arena unchanged
    with pytest.raises(RuntimeError, match="overflow"):
        a.peek(6)
    assert a.take(6) == base + 4 * rec and a.remaining == 0
    empty = _C.RankDataArena(0, 1 << 20)  # no buffer: nothing fits
    assert empty.capacity == 0 and not empty.fits(1)


def test_parity_band_matches_reference_definition():
    from b200ar.parallel.selector import parity_band

    rows = []
    for s, (ours, nccl) in {1: (10, 30), 2: (10, 10.5), 4: (10, 9.2), 8: (10, 8.0), 16: (10, 10.0)}.items():
        rows += [{"bytes": s, "impl": "custom", "us": ours}, {"bytes": s, "impl": "nccl", "us": nccl}]
    assert parity_band(rows) == [2, 4, 16]


def test_info_cli(capsys):
    from b200ar.__main__ import main

    assert main(["--json"]) == 0
    info = json.loads(capsys.readouterr().out)
    assert info["library"].startswith("_C") and set(info["selector"]) == {"2", "4", "8"}
    assert info["config"]["max_size"] > 0
    assert main([]) == 0
    assert "selector, 8 ranks" in capsys.readouterr().out


def test_attention_split_rule():
    from b200ar import _C

    for batch, hkv, max_len in ((1, 1, 2065), (8, 1, 2065), (32, 1, 2065), (64, 1, 2065), (4, 8, 4096),
                                (1, 1, 100), (512, 8, 2065)):
        s = _C.attention_splits(batch, hkv, max_len)
        assert 1 <= s <= 64
        # One wave of at most 3 CTAs per SM on 148 SMs (when the batch allows it).
        assert batch * hkv * s <= max(3 * 148, batch * hkv)
        # At least two 64-token chunks of cache per split.
        assert s == 1 or max_len // s >= 128
    assert _C.attention_splits(64, 1, 2065) == 6 and _C.attention_splits(1, 1, 2065) == 16


def test_skinny_split_rule():
    from b200ar import _C

    for n, k in ((1280, 8192), (7168, 8192), (8192, 3584), (8192, 1024), (128, 256)):
        s = _C.skinny_splits(n, k, 148)
        assert 1 <= s <= 16
        assert s == 1 or ((n + 127) // 128) * s <= 148


def test_reference_import_names_resolve_to_b200ar():
    import os
    import subprocess
    import sys

    import b200ar.shim

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    code = ("import pcie_allreduce, cuda_ipc\n"
            "from pcie_allreduce.cuda_ipc import CudaIPC\n"
            "import b200ar.compat as c\n"
            "assert pcie_allreduce.all_reduce is c.all_reduce and cuda_ipc.CudaIPC is CudaIPC\n"
            "assert sorted(pcie_allreduce.__all__) == sorted(c.__all__)\n"
            "assert pcie_allreduce.meta_size() == c.meta_size() > 0\n"
            "print('ok')\n")
    env = dict(os.environ, PYTHONPATH=os.pathsep.join([b200ar.shim.shim_path(), root]))
    res = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=300)
    assert res.returncode == 0 and res.stdout.strip().endswith("ok"), res.stderr[-2000:]


def _load_bench():
    import importlib.util
    import os

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    spec = importlib.util.spec_from_file_location("bench_main", os.path.join(root, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_bench_summary_rows_and_crossover():
    bench = _load_bench()
    sizes = bench.sizes(4096, 4 * 4096)
    assert sizes == [4096, 8192, 16384]
    per_call = {}
    for s in sizes:
        ours = 10.0 if s < 16384 else 40.0
        per_call[f"eager/{s}"] = [ours, ours + 1, ours + 2]
        per_call[f"graph/{s}"] = [ours - 1] * 3
        per_call[f"nccl_eager/{s}"] = [30.0] * 3
        per_call[f"nccl_graph/{s}"] = [30.0] * 3
    sweep, value, cross = bench.summarize(per_call, sizes, 8, lambda s: "lamport", True, True, True)
    assert [r["bytes"] for r in sweep] == sizes
    r0 = sweep[0]
    assert r0["eager_p50_us"] == 11.0 and r0["graph_p50_us"] == 9.0 and r0["nccl_eager_p50_us"] == 30.0
    assert r0["eager_us"] == {"p10": 10.2, "p50": 11.0, "p90": 11.8, "max": 12.0}
    assert r0["busbw_gbs"] == round(4096 / 11e-6 / 1e9 * 14 / 8, 1) and "busbw_frac_of_nvlink" in r0
    assert value == round((11.0 * 11.0 * 41.0) ** (1 / 3), 3)
    # NCCL is faster only at the largest size: that is the crossover.
    assert cross["crossover_bytes"] == {"eager": 16384, "graph": 16384}
    assert cross["crossover_band_bytes"]["eager"] == []
    sweep1, _, cross1 = bench.summarize({f"eager/{s}": [5.0] for s in sizes}, sizes, 1, str, False, False, False)
    assert cross1 == {} and "busbw_gbs" not in sweep1[0] and "graph_p50_us" not in sweep1[0]


def test_split_gate_up_layouts():
    from b200ar.ops.layers import ref_silu_mul, split_gate_up

    gu = torch.arange(2 * 256, dtype=torch.float32).view(2, 256)
    g, u = split_gate_up(gu, 64)
    assert torch.equal(g[0, :64], torch.arange(64.0)) and torch.equal(u[0, :64], torch.arange(64.0, 128.0))
    assert torch.equal(g[1, 64:], torch.arange(256 + 128, 256 + 192.0))
    g0, u0 = split_gate_up(gu, 0)
    assert torch.equal(g0, gu[:, :128]) and torch.equal(u0, gu[:, 128:])
    assert ref_silu_mul(gu.to(torch.bfloat16), 64).shape == (2, 128)


def test_plan_ctas_never_exceeds_coresident_count():
    """Barrier kernels wait on the same CTA index of every peer, so a launch
    must never have more CTAs than fit on the device at once."""
    from b200ar._native import _C

    V = _C.VARIANTS
    barrier_kernels = ["oneshot_push", "oneshot_pull", "twoshot", "registered", "lamport", "nvls"]
    sizes = [16, 4096, 1 << 20, 64 << 20, 1 << 30]
    for name in barrier_kernels:
        for world in range(2, 9):
            for resident in (1, 37, 148, 296):
                for requested in (0, 1, 100, 444, 512):
                    for nbytes in sizes:
                        c = _C.plan_ctas(V[name], nbytes, world, requested, resident)
                        assert 1 <= c <= min(resident, _C.MAX_CTAS), (name, world, resident, requested, nbytes, c)
                        if requested:
                            assert c == min(requested, resident)
    # Large messages want more CTAs than one SM's worth; the clamp decides.
    assert _C.plan_ctas(V["twoshot"], 1 << 30, 8, 0, 148) == 148
    assert _C.plan_ctas(V["copy"], 1 << 20, 1, 0, 148) == 0 and _C.plan_ctas(V["nccl"], 1 << 20, 8, 0, 148) == 0


def test_bench_compact_rows():
    bench = _load_bench()
    sweep = [{"bytes": 4096, "variant": "lamport", "eager_p50_us": 11.0, "graph_p50_us": 9.0,
              "nccl_eager_p50_us": 20.0, "eager_us": {}},
             {"bytes": 8192, "variant": "twoshot", "eager_p50_us": 12.0}]
    rows = bench.compact_rows(sweep, {4096: 40.123})
    assert bench.ROW_COLS[0] == "bytes" and len(bench.ROW_COLS) == 7
    assert rows == [[4096, "lamport", 11.0, 9.0, 20.0, None, 40.12], [8192, "twoshot", 12.0, None, None, None, None]]


def test_partial_sweep_table_merge():
    from b200ar.parallel.selector import merge_partial_table

    old = [(16384, "lamport", 1), (131072, "lamport", 16), (4194304, "lamport", 296), (1 << 62, "twoshot", 64)]
    new = [(2097152, "lamport", 64), (1 << 62, "twoshot_push", 148)]
    got = merge_partial_table(old, new, 1 << 20)
    assert got == [(16384, "lamport", 1), (131072, "lamport", 16), (524288, "lamport", 296),
                   (2097152, "lamport", 64), (1 << 62, "twoshot_push", 148)]
