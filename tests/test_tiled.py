"""The column-blocked B = 1 tick (nsb_dendritic_step_tiled) against the oracle."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from _util import OracleMatrix, assert_same_as, bench_model, csr_of, make, npy, params_of
from neurosim_gpu_b200 import (NativeDendriticMatrixRuntime, encode_sparse_weights,
                               load_native_extension, quantize_dequantize, random_topology)
from neurosim_gpu_b200 import native
from neurosim_gpu_b200.tiled import build_tiled_layout, emulate


def _packed(graph, fmt):
    if fmt == "fp32":
        return graph.in_weight, None, None, graph.in_weight
    if fmt == "fp16":
        return graph.in_weight.half(), None, None, graph.in_weight.half().float()
    codes, scales, scale = encode_sparse_weights(graph.in_weight, fmt)
    return codes, scales, scale, quantize_dequantize(graph.in_weight, fmt)


def _smem_bytes():
    lib = native.load_library()
    return lambda cols, bufs: int(lib.nsb_tiled_smem_bytes(cols, bufs))


@pytest.mark.parametrize("chunk", [None, 4, 8, 16])
@pytest.mark.parametrize("fmt", ["fp32", "fp16", "fp8", "nvfp4"])
@pytest.mark.parametrize("n,m,ctas,smem", [(97, 600, 4, 232448), (2000, 60000, 8, 8000),
                                           (5000, 100000, 16, 6000), (3001, 40001, 5, 232448),
                                           (5000, 100000, 2, 6000), (1, 0, 3, 232448),
                                           (300, 9000, 148, 232448), (2000, 200000, 8, 232448)])
def test_layout_emulation_matches_oracle_cpu(fmt, n, m, ctas, smem, chunk):
    """The layout builder alone, emulated on CPU (no GPU needed), at each
    chunk width (None: the builder's choice from the mean piece length; 16
    slots only for the 1-byte and half-byte weight formats)."""
    if chunk == 16 and fmt not in ("fp8", "nvfp4"):
        pytest.skip("16-slot chunks are for E4M3 / NVFP4 weights")
    graph = random_topology(n, m, device="cpu", seed=3)
    weight, scales, scale, decoded = _packed(graph, fmt)
    layout = build_tiled_layout(graph.in_rowptr, graph.in_col, weight, neurons=n, ctas=ctas,
                                smem_limit=smem, block_scales=scales, global_scale=scale,
                                smem_bytes=_smem_bytes(), chunk=chunk)
    assert chunk is None or layout.chunk == chunk
    assert layout.n_slots % (32 * layout.chunk) == 0
    x = torch.rand(1, n, generator=torch.Generator().manual_seed(1))
    want = oracle.spmv(csr_of(graph, decoded), npy(x))[0]
    np.testing.assert_allclose(emulate(layout, x).numpy(), want, atol=1e-6, rtol=0)
    assert layout.n_slots >= graph.n_edges


@pytest.mark.gpu
@pytest.mark.parametrize("chunk", [4, 8, 16])
@pytest.mark.parametrize("fmt", ["fp32", "fp16", "fp8", "nvfp4"])
@pytest.mark.parametrize("n,m,ctas,smem", [(97, 600, 4, 232448), (2000, 60000, 8, 8000),
                                           (5000, 100000, 16, 6000), (3001, 40001, 5, 232448),
                                           (20000, 400000, 148, 24000), (5000, 100000, 2, 6000),
                                           (2000, 200000, 8, 232448)])
def test_tiled_tick_matches_oracle(fmt, n, m, ctas, smem, chunk):
    if chunk == 16 and fmt not in ("fp8", "nvfp4"):
        pytest.skip("16-slot chunks are for E4M3 / NVFP4 weights")
    ext = load_native_extension()
    graph = random_topology(n, m, device="cpu", seed=3).to("cuda")
    weight, scales, scale, decoded = _packed(graph, fmt)
    layout = build_tiled_layout(graph.in_rowptr, graph.in_col, weight, neurons=n, ctas=ctas,
                                smem_limit=smem, block_scales=scales, global_scale=scale,
                                chunk=chunk)
    model = bench_model(n)
    state = torch.rand(1, n, generator=torch.Generator().manual_seed(2)).cuda()
    dendrite = torch.rand(1, n, generator=torch.Generator().manual_seed(4)).cuda() - 0.5
    adaptation = torch.rand(1, n, generator=torch.Generator().manual_seed(5)).cuda()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    # product
    got = ext.tiled_propagate(layout, state, status=status)
    want = oracle.spmv(csr_of(graph, decoded), npy(state))
    np.testing.assert_allclose(npy(got), want, atol=2e-6, rtol=0)
    # tick
    s, d, a = ext.dendritic_step_tiled(state, dendrite, adaptation, model.parameters(), layout,
                                       None, 0.2, None, 0.1, status=status)
    ws, wd, wa = oracle.matrix_tick(csr_of(graph, decoded), npy(state), npy(dendrite),
                                    npy(adaptation), [npy(p) for p in model.parameters()], 0.2, 0.1)
    for got, want in ((s, ws), (d, wd), (a, wa)):
        np.testing.assert_allclose(npy(got), want, atol=2e-6, rtol=0)
    assert int(status.item()) == 0


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", ["fp32", "nvfp4"])
def test_runtime_uses_tiled_path_for_single_batch(fmt):
    graph, model, state = make(3000, 1, 90000)
    tiled = NativeDendriticMatrixRuntime(graph, model, state.clone(), precision=fmt,
                                         kernel="tiled")
    csr = NativeDendriticMatrixRuntime(graph, model, state.clone(), precision=fmt, kernel="csr")
    decoded = quantize_dequantize(graph.in_weight, fmt)
    reference = OracleMatrix(graph, model, state, weight=decoded)
    with torch.inference_mode():
        for _ in range(20):
            tiled.step(0.2, dendritic_drive=0.1)
            csr.step(0.2, dendritic_drive=0.1)
            reference.step(0.2, 0.1)
        tiled.run(45, 0.2, dendritic_drive=0.1, graph_ticks=16)
        csr.run(45, 0.2, dendritic_drive=0.1, graph_ticks=16)
    for _ in range(45):
        reference.step(0.2, 0.1)
    assert tiled.kernel_path == "tiled" and csr.kernel_path == "csr"
    assert_same_as(tiled, reference, atol=2e-6)
    assert_same_as(tiled, csr, atol=2e-6)
    tiled.check_status()


@pytest.mark.gpu
def test_tiled_rejects_bad_inputs():
    ext = load_native_extension()
    graph, model, state = make(500, 2, 5000)
    layout = build_tiled_layout(graph.in_rowptr, graph.in_col, graph.in_weight, neurons=500,
                                ctas=4, smem_limit=232448)
    with pytest.raises(RuntimeError, match="B = 1"):
        ext.dendritic_step_tiled(state, state, state, model.parameters(), layout, None, 0.,
                                 None, 0.)
    one = state[:1].contiguous()
    with pytest.raises(RuntimeError, match="aligned"):
        odd = torch.zeros(1, 501, device="cuda")[:, 1:]
        ext.dendritic_step_tiled(odd, one, one, model.parameters(), layout, None, 0., None, 0.)


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", ["fp32", "nvfp4"])
def test_multi_tick_run_equals_single_ticks_bitwise(fmt):
    """nsb_dendritic_run_tiled (one persistent launch) == repeated nsb_dendritic_step_tiled."""
    ext = load_native_extension()
    graph = random_topology(6000, 150000, device="cpu", seed=11).to("cuda")
    weight, scales, scale, _ = _packed(graph, fmt)
    layout = build_tiled_layout(graph.in_rowptr, graph.in_col, weight, neurons=6000, ctas=24,
                                smem_limit=12000, block_scales=scales, global_scale=scale)
    assert layout.blocks > 1
    model = bench_model(6000)
    s0 = torch.rand(1, 6000, generator=torch.Generator().manual_seed(2)).cuda()
    d0 = torch.zeros_like(s0)
    a0 = torch.zeros_like(s0)
    drive = torch.rand(1, 6000, generator=torch.Generator().manual_seed(9)).cuda() * 0.4
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    s, d, a = s0, d0, a0
    for _ in range(17):
        s, d, a = ext.dendritic_step_tiled(s, d, a, model.parameters(), layout, drive, 0.0,
                                           None, 0.1, status=status)
    out = [torch.empty_like(s0) for _ in range(3)]
    ext.prepare_step_tiled(s0, d0, a0, model.parameters(), layout, drive, 0.0, None, 0.1,
                           out=out, status=status, ticks=17)()
    torch.cuda.synchronize()
    for got, want in zip(out, (s, d, a)):
        assert torch.equal(got, want)
    assert int(status.item()) == 0
    assert int(layout.workspace()[256:].count_nonzero().item()) == 0  # row sums left cleared


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", ["fp32", "fp8"])
def test_rollout_per_tick_drives_and_history_match_single_ticks_and_oracle(fmt):
    """nsb_dendritic_rollout_tiled: tick k reads drive row k and writes history
    row k; bit-equal to single ticks with those drives, and to the oracle."""
    ext = load_native_extension()
    n, ticks = 6000, 13
    graph = random_topology(n, 150000, device="cpu", seed=12).to("cuda")
    weight, scales, scale, decoded = _packed(graph, fmt)
    layout = build_tiled_layout(graph.in_rowptr, graph.in_col, weight, neurons=n, ctas=24,
                                smem_limit=12000, block_scales=scales, global_scale=scale)
    model = bench_model(n)
    gen = torch.Generator().manual_seed(4)
    s0 = torch.rand(1, n, generator=gen).cuda()
    d0 = (torch.rand(1, n, generator=gen) - 0.5).cuda()
    a0 = torch.rand(1, n, generator=gen).cuda()
    # Drive rows 5 floats apart in a wider buffer: the tick stride is not N.
    stride = n + 5
    drives = (torch.rand(ticks * stride, generator=gen) * 0.4).cuda()
    drive_row = [drives[k * stride: k * stride + n].view(1, n) for k in range(ticks)]
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    s, d, a = s0, d0, a0
    singles = []
    for k in range(ticks):
        s, d, a = ext.dendritic_step_tiled(s, d, a, model.parameters(), layout, drive_row[k], 0.0,
                                           None, 0.1, status=status)
        singles.append(s)
    out = [torch.empty_like(s0) for _ in range(3)]
    history = torch.full((ticks, 1, n), float("nan"), device="cuda")
    ext.prepare_step_tiled(s0, d0, a0, model.parameters(), layout, drive_row[0], 0.0, None, 0.1,
                           out=out, status=status, ticks=ticks, rollout=(stride, history))()
    torch.cuda.synchronize()
    for got, want in zip(out, (s, d, a)):
        assert torch.equal(got, want)
    for k in range(ticks):
        assert torch.equal(history[k], singles[k]), k
    assert int(status.item()) == 0
    # Against the oracle on the decoded weights.
    csr, params = csr_of(graph, decoded), params_of(model)
    os_, od, oa = npy(s0), npy(d0), npy(a0)
    for k in range(ticks):
        os_, od, oa = oracle.matrix_tick(csr, os_, od, oa, params, npy(drive_row[k]),
                                         np.full_like(os_, 0.1))
        np.testing.assert_allclose(npy(history[k]), os_, atol=1e-5, rtol=0)
    # Without a history and with a zero drive stride it is the plain multi-tick run.
    plain = [torch.empty_like(s0) for _ in range(3)]
    ext.prepare_step_tiled(s0, d0, a0, model.parameters(), layout, drive_row[0], 0.0, None, 0.1,
                           out=plain, status=status, ticks=5)()
    rolled = [torch.empty_like(s0) for _ in range(3)]
    ext.prepare_step_tiled(s0, d0, a0, model.parameters(), layout, drive_row[0], 0.0, None, 0.1,
                           out=rolled, status=status, ticks=5, rollout=(0, None))()
    torch.cuda.synchronize()
    for got, want in zip(rolled, plain):
        assert torch.equal(got, want)


@pytest.mark.gpu
def test_in_kernel_decoders_exhaustive():
    """Every E4M3 code and every (E2M1 code, E4M3 block scale) pair decodes to the
    reference quantizer's dequantized value, bit for bit (one edge per row, source 1)."""
    from neurosim_gpu_b200.precision import e2m1_to_float, e4m3_to_float
    ext = load_native_extension()
    g = torch.tensor([0.0371], device="cuda")
    # E4M3: 256 rows, row i has one edge of code i.
    n = 256
    rowptr = torch.arange(n + 1, dtype=torch.int32, device="cuda")
    col = torch.arange(n, dtype=torch.int32, device="cuda")
    codes = torch.arange(n, dtype=torch.uint8, device="cuda")
    layout = build_tiled_layout(rowptr, col, codes, neurons=n, ctas=4, smem_limit=232448,
                                global_scale=g)
    got = ext.tiled_propagate(layout, torch.ones(1, n, device="cuda"))
    want = e4m3_to_float(codes) * g
    np.testing.assert_array_equal(npy(got)[0], npy(want))
    # NVFP4: 4096 rows; edge e has E2M1 code e % 16 and lies in block e // 16 with scale code e // 16.
    n = 4096
    rowptr = torch.arange(n + 1, dtype=torch.int32, device="cuda")
    col = torch.arange(n, dtype=torch.int32, device="cuda")
    nib = torch.arange(n, device="cuda") % 16
    packed = (nib[0::2] | (nib[1::2] << 4)).to(torch.uint8)
    scales = torch.arange(256, dtype=torch.uint8, device="cuda")
    layout = build_tiled_layout(rowptr, col, packed, neurons=n, ctas=8, smem_limit=232448,
                                block_scales=scales, global_scale=g)
    got = ext.tiled_propagate(layout, torch.ones(1, n, device="cuda"))
    want = e2m1_to_float(nib.to(torch.uint8)) * (e4m3_to_float(scales).repeat_interleave(16) * g)
    np.testing.assert_array_equal(npy(got)[0], npy(want))


def test_sharded_layouts_split_rows_like_the_whole_graph_cpu():
    """Split points depend only on the graph, not on which rows a layout holds
    (a graph dense enough for split sub-tasks: ~55 edges per row piece)."""
    n, m = 9001, 2000000
    graph = random_topology(n, m, device="cpu", seed=6)
    rowptr = graph.in_rowptr.long()
    smem = _smem_bytes()
    whole = build_tiled_layout(graph.in_rowptr, graph.in_col, graph.in_weight, neurons=n, ctas=20,
                               smem_limit=12000, smem_bytes=smem)
    assert whole.splits > 1
    for lo, hi in ((0, 4501), (4501, 9001)):
        e0, e1 = int(rowptr[lo]), int(rowptr[hi])
        part = build_tiled_layout((rowptr[lo:hi + 1] - e0).to(torch.int32),
                                  graph.in_col[e0:e1].contiguous(), graph.in_weight[e0:e1],
                                  neurons=hi - lo, cols=n, ctas=20, smem_limit=12000,
                                  smem_bytes=smem)
        assert (part.blocks, part.block_cols, part.split_chunks) == \
            (whole.blocks, whole.block_cols, whole.split_chunks)



@pytest.mark.parametrize("first,cap", [(1, 32), (2, 32), (128, 128)])
def test_rollout_chunks_cover_the_ticks_and_ramp_cpu(first, cap):
    """Streamed-rollout launch lengths add up to the ticks and none exceeds the
    cap; a head doubling from ``first`` (while below the cap) opens the
    rollout, the same head in reverse closes it, and the middle launches
    differ by at most one tick."""
    from neurosim_gpu_b200.tiled import rollout_chunks
    if first == 1:
        assert rollout_chunks(20, cap, first) == [1, 2, 4, 6, 4, 2, 1]
        assert rollout_chunks(512, cap, first)[:6] == [1, 2, 4, 8, 16, 30]
    for ticks in list(range(1, 200)) + [512, 1000, 4099]:
        chunks = rollout_chunks(ticks, cap, first)
        assert sum(chunks) == ticks and all(0 < c <= max(cap, first) for c in chunks)
        head, size = [], first
        while size < cap and 2 * (sum(head) + size) <= ticks:
            head.append(size)
            size *= 2
        assert chunks[:len(head)] == head and chunks[len(chunks) - len(head):] == head[::-1]
        middle = chunks[len(head):len(chunks) - len(head)]
        assert not middle or max(middle) - min(middle) <= 1, (ticks, chunks)


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", ["fp32", "nvfp4"])
@pytest.mark.parametrize("rows_per_cta", [None, 40])
def test_staged_update_equals_direct_update_bitwise(fmt, rows_per_cta):
    """The update after the grid barrier reads its operands through shared
    memory (bulk copies, when every operand is a contiguous 16-byte aligned
    vector) or straight from L2 (strided parameters): same states bit for bit,
    over several ticks of one launch and with more rows per CTA than one
    staged chunk holds (small shared memory: the rows go in several chunks)."""
    ext = load_native_extension()
    n = 8000  # a multiple of 4
    graph = random_topology(n, 240000, device="cpu", seed=21).to("cuda")
    weight, scales, scale, _ = _packed(graph, fmt)
    smem = 232448 if rows_per_cta is None else 12000
    layout = build_tiled_layout(graph.in_rowptr, graph.in_col, weight, neurons=n,
                                ctas=8 if rows_per_cta is None else n // rows_per_cta // 25,
                                smem_limit=smem, block_scales=scales, global_scale=scale)
    model = bench_model(n)
    contiguous = [p.contiguous().clone() for p in model.parameters()]
    strided = [torch.empty(2 * n, device="cuda")[::2].copy_(p) for p in contiguous]
    s0 = torch.rand(1, n, generator=torch.Generator().manual_seed(5)).cuda()
    results = []
    for params in (contiguous, strided):
        out = [torch.empty_like(s0) for _ in range(3)]
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        ext.prepare_step_tiled(s0, torch.zeros_like(s0), torch.zeros_like(s0), params, layout,
                               None, 0.2, None, 0.1, out=out, status=status, ticks=9)()
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        results.append(out)
    for got, want in zip(*results):
        assert torch.equal(got, want)


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", ["fp32", "fp16", "fp8", "nvfp4"])
@pytest.mark.parametrize("n,m,smem", [(6000, 400000, 232448), (6000, 150000, 12000)])
def test_chunk_widths_tick_bit_identically(fmt, n, m, smem):
    """A lane sums its piece in CSR order whatever the chunk width, and splits
    cut pieces at the same edges, so 4- and 8-slot layouts tick bit for bit
    alike (20 ticks in one persistent launch)."""
    ext = load_native_extension()
    graph = random_topology(n, m, device="cpu", seed=12).to("cuda")
    weight, scales, scale, _ = _packed(graph, fmt)
    model = bench_model(n)
    s0 = torch.rand(1, n, generator=torch.Generator().manual_seed(2)).cuda()
    results = []
    for chunk in (4, 8, 16) if fmt in ("fp8", "nvfp4") else (4, 8):
        layout = build_tiled_layout(graph.in_rowptr, graph.in_col, weight, neurons=n, ctas=24,
                                    smem_limit=smem, block_scales=scales, global_scale=scale,
                                    chunk=chunk)
        assert layout.chunk == chunk
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        out = [torch.empty_like(s0) for _ in range(3)]
        ext.prepare_step_tiled(s0, torch.zeros_like(s0), torch.zeros_like(s0), model.parameters(),
                               layout, None, 0.2, None, 0.1, out=out, status=status, ticks=20)()
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        results.append(out)
    for other in results[1:]:
        for a, b in zip(results[0], other):
            assert torch.equal(a, b)
