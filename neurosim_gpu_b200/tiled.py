"""Column-blocked ("tiled") layout of a destination CSR for the B = 1 tick.

The layout re-arranges the edges of ``W[dst, src]`` (``in_rowptr``, ``in_col``
and the weights in any storage format) so that the tick kernel
(``nsb_dendritic_step_tiled``) can keep the gathered source state in shared
memory:

* CTA ``c`` (one per SM) owns destination rows ``[row_begin[c], row_begin[c+1])``,
  cut so every CTA holds about the same number of edges plus rows.
* Columns are split into ``blocks`` blocks of ``block_cols`` columns; one block
  of the state fits in shared memory (two when ``buffers == 2``).
* For each CTA and block, the rows' pieces (their edges inside the block, a
  contiguous run of the original CSR row) are sorted by length and grouped 32 at
  a time into tasks.  In a task, lane ``i`` owns one row and its ``j``-th edge
  sits at slot ``task_offset + 32 j + i``: a warp's load covers 32 consecutive
  slots.  Shorter pieces are padded to the task length with column
  ``block_cols`` (a zero in shared memory) and weight 0.

Edge order inside a row piece is the CSR order, so the sums equal a
sequential dot product per (row, block) followed by a sum over blocks.
The builder runs on the weights' device with PyTorch ops; it is cached by the
runtime per ``weight_version``.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import native

LANES = 32
MAX_CTA_ROWS = 32767  # row ids are int16 inside a CTA


@dataclass
class TiledLayout:
    neurons: int          # destination rows of this layout
    n_edges: int
    ctas: int
    blocks: int
    block_cols: int
    buffers: int
    max_rows: int
    format: int
    row_begin: torch.Tensor
    task_ptr: torch.Tensor
    task_offset: torch.Tensor
    task_len: torch.Tensor
    task_rows: torch.Tensor
    task_orig: torch.Tensor | None
    col: torch.Tensor
    weight: torch.Tensor
    block_scales: torch.Tensor | None
    global_scale: torch.Tensor | None
    cols: int = 0         # length of the gathered source vector (0: same as neurons)

    def __post_init__(self) -> None:
        if self.cols == 0:
            self.cols = self.neurons

    @property
    def n_tasks(self) -> int:
        return self.task_len.numel()

    @property
    def n_slots(self) -> int:
        return self.col.numel()

    @property
    def padding_fraction(self) -> float:
        return 1.0 - self.n_edges / max(self.n_slots, 1)

    def stream_bytes(self) -> int:
        """Bytes one tick streams from this layout (indices, weights, task tables)."""
        tables = sum(t.numel() * t.element_size() for t in (
            self.row_begin, self.task_ptr, self.task_offset, self.task_len, self.task_rows))
        if self.task_orig is not None:
            tables += self.task_orig.numel() * 4
        return self.col.numel() * 4 + self.weight.numel() * self.weight.element_size() + tables

    def c_struct(self) -> "native._TiledLayout":
        def ptr(t):
            return t.data_ptr() if t is not None and t.numel() else None
        return native._TiledLayout(
            self.ctas, self.blocks, self.block_cols, self.buffers, self.max_rows, self.format,
            self.n_tasks, self.n_slots,
            self.block_scales.numel() if self.block_scales is not None else 0, self.cols,
            ptr(self.row_begin), ptr(self.task_ptr), ptr(self.task_offset), ptr(self.task_len),
            ptr(self.task_rows), ptr(self.task_orig), ptr(self.col), ptr(self.weight),
            ptr(self.block_scales), ptr(self.global_scale))


def plan_blocks(neurons: int, max_rows: int, smem_limit: int, smem_bytes) -> tuple[int, int, int]:
    """(blocks, block_cols, buffers) that fit one CTA's shared memory."""
    whole = -(-neurons // 4) * 4
    if smem_bytes(whole, max_rows, 1) <= smem_limit:
        return 1, whole, 1
    per_buffer = (smem_limit - smem_bytes(0, max_rows, 2)) // 8 - 4
    cap = (per_buffer // LANES) * LANES
    if cap < LANES:
        raise ValueError("shared memory too small for a tiled layout")
    blocks = -(-neurons // cap)
    block_cols = -(-(-(-neurons // blocks)) // LANES) * LANES
    return blocks, block_cols, 2


def cta_row_ranges(rowptr: torch.Tensor, ctas: int) -> torch.Tensor:
    """Row boundaries that give every CTA about (edges + rows) / ctas work."""
    n = rowptr.numel() - 1
    cost = rowptr.long() + torch.arange(n + 1, device=rowptr.device)
    total = int(cost[-1])
    targets = torch.arange(ctas + 1, device=rowptr.device, dtype=torch.int64) * total // ctas
    begin = torch.searchsorted(cost, targets)
    begin[0] = 0
    begin[-1] = n
    return torch.cummax(begin, 0).values


def build_tiled_layout(in_rowptr: torch.Tensor, in_col: torch.Tensor, weight: torch.Tensor,
                       *, neurons: int, ctas: int, smem_limit: int, block_scales=None,
                       global_scale=None, smem_bytes=None, cols: int | None = None,
                       scale_offset: int = 0) -> TiledLayout:
    """Build the tiled layout of one graph.

    ``weight`` is the CSR value array in its storage format (float32 / float16 /
    uint8 E4M3 codes / uint8 packed NVFP4).  ``neurons`` is the number of
    destination rows (``in_rowptr`` has neurons + 1 entries, starting at 0);
    ``cols`` is the length of the gathered source (default: ``neurons``).  For a
    block of rows cut out of a larger NVFP4 CSR, ``scale_offset`` is the CSR
    position of the block's first edge (it selects the original block scales).
    """
    device = in_col.device
    if smem_bytes is None:
        lib = native.load_library()
        smem_bytes = lambda cols, rows, bufs: int(lib.nsb_tiled_smem_bytes(cols, rows, bufs))  # noqa: E731
    n, m = neurons, in_col.numel()
    cols = n if cols is None else cols
    if block_scales is not None:
        fmt = native.NVFP4
    elif weight.dtype == torch.uint8:
        fmt = native.E4M3
    elif weight.dtype == torch.float16:
        fmt = native.F16
    else:
        fmt = native.F32
    rowptr = in_rowptr.to(torch.int64)
    row_begin = cta_row_ranges(rowptr, ctas)
    rows_per_cta = row_begin[1:] - row_begin[:-1]
    max_rows = int(rows_per_cta.max())
    if max_rows > MAX_CTA_ROWS:
        raise ValueError("too many rows per CTA for the tiled layout")
    blocks, block_cols, buffers = plan_blocks(cols, max_rows, smem_limit, smem_bytes)

    degree = rowptr[1:] - rowptr[:-1]
    row_of_edge = torch.repeat_interleave(torch.arange(n, device=device), degree)
    col64 = in_col.to(torch.int64)
    block_of_edge = col64 // block_cols
    piece = row_of_edge * blocks + block_of_edge                       # (row, block) pair id
    piece_len = torch.bincount(piece, minlength=n * blocks).view(n, blocks)
    piece_start = rowptr[:-1, None] + torch.cumsum(piece_len, 1) - piece_len

    # Sort (row, block) pairs by (CTA, block), then by piece length (longest first).
    cta_of_row = torch.searchsorted(row_begin, torch.arange(n, device=device), right=True) - 1
    group = (cta_of_row[:, None] * blocks + torch.arange(blocks, device=device)).flatten()
    lengths = piece_len.flatten()
    order = torch.sort(-lengths, stable=True).indices
    order = order[torch.sort(group[order], stable=True).indices]
    sorted_group = group[order]
    group_size = torch.bincount(sorted_group, minlength=ctas * blocks)
    group_start = torch.cumsum(group_size, 0) - group_size
    position = torch.arange(order.numel(), device=device) - group_start[sorted_group]
    tasks_per_group = (group_size + LANES - 1) // LANES
    task_ptr = torch.zeros(ctas * blocks + 1, dtype=torch.int64, device=device)
    torch.cumsum(tasks_per_group, 0, out=task_ptr[1:])
    pair_task = task_ptr[sorted_group] + position // LANES
    pair_lane = position % LANES
    n_tasks = int(task_ptr[-1])
    task_len = torch.zeros(n_tasks, dtype=torch.int64, device=device)
    task_len.scatter_reduce_(0, pair_task, lengths[order], reduce="amax")
    task_offset = torch.cumsum(task_len * LANES, 0) - task_len * LANES
    slots = int((task_len * LANES).sum())
    if slots >= 2**31:
        raise ValueError("tiled layout exceeds 2^31 slots")
    pair_row = order // blocks
    task_rows = torch.full((n_tasks, LANES), -1, dtype=torch.int16, device=device)
    task_rows[pair_task, pair_lane] = (pair_row - row_begin[cta_of_row[pair_row]]).to(torch.int16)

    # Slot of every edge: its pair's task and lane, and its rank inside the piece.
    rank_of_pair = torch.empty_like(order)
    rank_of_pair[order] = torch.arange(order.numel(), device=device)
    r = rank_of_pair[piece]
    within = torch.arange(m, device=device) - piece_start.flatten()[piece]
    slot = task_offset[pair_task[r]] + within * LANES + pair_lane[r]
    col = torch.full((slots,), block_cols, dtype=torch.int32, device=device)
    col[slot] = (col64 - block_of_edge * block_cols).to(torch.int32)

    task_orig = None
    if fmt == native.NVFP4:
        nibbles = torch.stack((weight & 15, weight >> 4), dim=1).flatten()[:m]
        codes = torch.zeros(slots, dtype=torch.uint8, device=device)
        codes[slot] = nibbles
        tiled_weight = (codes[0::2] | (codes[1::2] << 4)).contiguous()
        task_orig = torch.zeros((n_tasks, LANES), dtype=torch.int32, device=device)
        task_orig[pair_task, pair_lane] = (piece_start.flatten()[order] + scale_offset).to(torch.int32)
    else:
        tiled_weight = torch.zeros(slots, dtype=weight.dtype, device=device)
        tiled_weight[slot] = weight
    return TiledLayout(
        neurons=n, n_edges=m, ctas=ctas, blocks=blocks, block_cols=block_cols, buffers=buffers,
        max_rows=max_rows, format=fmt, row_begin=row_begin.to(torch.int32),
        task_ptr=task_ptr.to(torch.int32), task_offset=task_offset.to(torch.int32),
        task_len=task_len.to(torch.int32), task_rows=task_rows.contiguous(), task_orig=task_orig,
        col=col, weight=tiled_weight, block_scales=block_scales, global_scale=global_scale,
        cols=cols)


def emulate(layout: TiledLayout, source: torch.Tensor) -> torch.Tensor:
    """What the kernel computes, j = W @ source (B = 1), in float64 on any device.

    Used by the tests to check a layout without a GPU.
    """
    x = source.reshape(-1).double()
    out = torch.zeros(layout.neurons, dtype=torch.float64, device=x.device)
    w = _decoded_slots(layout).double()
    blocks_of_task = torch.repeat_interleave(
        torch.arange(layout.ctas * layout.blocks, device=x.device),
        (layout.task_ptr[1:] - layout.task_ptr[:-1]).long())
    cta = blocks_of_task // layout.blocks
    block = blocks_of_task % layout.blocks
    out = torch.zeros(layout.neurons, dtype=torch.float64, device=x.device)
    padded = torch.cat([x, torch.zeros(layout.blocks * layout.block_cols + 1 - x.numel(),
                                       dtype=x.dtype, device=x.device)])
    for q in range(layout.n_tasks):
        length = int(layout.task_len[q])
        if length == 0:
            continue
        base = int(layout.task_offset[q])
        cols = layout.col[base: base + length * LANES].view(length, LANES).long()
        vals = w[base: base + length * LANES].view(length, LANES)
        start = int(block[q]) * layout.block_cols
        gathered = torch.where(cols == layout.block_cols, torch.zeros_like(vals),
                               padded[(start + cols).clamp(max=padded.numel() - 1)])
        dots = (vals * gathered).sum(0)
        rows = layout.task_rows[q].long()
        keep = rows >= 0
        out[(int(layout.row_begin[cta[q]]) + rows[keep])] += dots[keep]
    return out


def _decoded_slots(layout: TiledLayout) -> torch.Tensor:
    if layout.format == native.F32 or layout.format == native.F16:
        return layout.weight.float()
    from .precision import e4m3_to_float, e2m1_to_float
    if layout.format == native.E4M3:
        return e4m3_to_float(layout.weight) * layout.global_scale.float()
    codes = torch.stack((layout.weight & 15, layout.weight >> 4), dim=1).flatten()
    slots = torch.arange(codes.numel(), device=codes.device)
    task = torch.searchsorted(layout.task_offset.long(), slots, right=True) - 1
    j = (slots - layout.task_offset.long()[task]) // LANES
    lane = slots % LANES
    orig = layout.task_orig.long()[task, lane] + j
    block = orig.clamp(max=layout.block_scales.numel() * 16 - 1) // 16
    factor = e4m3_to_float(layout.block_scales[block]) * layout.global_scale.float()
    return e2m1_to_float(codes) * factor


def smem_limit(device: torch.device) -> int:
    """Opt-in shared memory per block of ``device``."""
    props = torch.cuda.get_device_properties(device)
    return int(getattr(props, "shared_memory_per_block_optin", 232448))


def sm_count(device: torch.device) -> int:
    return int(torch.cuda.get_device_properties(device).multi_processor_count)


def status_word(device: torch.device) -> torch.Tensor:
    return torch.zeros(1, dtype=torch.int32, device=device)


__all__ = ["TiledLayout", "build_tiled_layout", "emulate", "plan_blocks", "cta_row_ranges",
           "smem_limit", "sm_count", "status_word", "ctypes"]
