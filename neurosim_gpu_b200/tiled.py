"""Column-blocked ("tiled") layout of a destination CSR for the B = 1 tick.

The layout re-arranges the edges of ``W[dst, src]`` (``in_rowptr``, ``in_col``
and the weights in any storage format) so that the tick kernel
(``nsb_dendritic_step_tiled``) keeps the gathered source state in shared memory
and streams the edges with vector loads:

* The gathered columns are split into ``blocks`` blocks of ``block_cols``
  columns, each small enough to sit in one CTA's shared memory.
* A *stage* is one column block and a contiguous range of destination rows.
  When there are at least as many CTAs as blocks, every CTA runs exactly one
  stage: block ``k`` gets a share of the CTAs proportional to its edges, and
  its rows are cut into that many ranges of about equal edge count.  The state
  block is then staged once per tick.  (With more blocks than CTAs, CTA ``c``
  runs the full-row stages of blocks ``c, c + ctas, ...``, double-buffered.)
* For each stage, the rows' non-empty pieces (their edges inside the block, a
  contiguous run of the original CSR row) are sorted by chunk count (then by
  row) and grouped 32 at a time into tasks.  A chunk is ``K`` slots per lane
  (``chunk``: 4, or 8 when the pieces average at least WIDE_CHUNK_MIN_EDGES
  edges); a task has ``chunks`` chunks, lane ``i`` owns one row and its edge
  ``j`` sits at slot ``first + 32K * (j // K) + K * i + j % K``, so one lane
  reads K edges with one vector load of columns and one of weights and a
  warp's loads cover 32K consecutive slots.  Shorter pieces are padded with
  column ``block_cols`` (a zero in shared memory) and weight 0.  A lane sums
  its piece in CSR order whatever K is.  Consecutive groups of one stage with
  the same chunk count are merged into tasks of several such segments (up to
  MERGE_SLOTS slots per lane; fp32 only), each segment's 32 rows being one
  row group of ``task_rows``.
* Columns are stored relative to their block as uint16 (2 bytes per edge
  instead of the CSR's 4).
* A task is cut into sub-tasks of ``split_chunks`` chunks (edges
  ``K * split_chunks * h ...`` of every lane's piece form split ``h``; the
  split is a whole number of edges, SPLIT_EDGES, for either K), so the
  CTA's work comes in pieces small enough to balance over its warps.  Each
  sub-task's per-row sums go to a workspace plane ``part[block][h][row]``;
  after a grid-wide barrier every CTA adds the planes of its share of the rows
  in (block, split) order and applies the pointwise update.  The split points
  depend only on a row's own piece, not on how rows are grouped into tasks.
* NVFP4: codes are re-packed two per byte by slot.  Each task carries a table
  of uint16 scale pairs (for lane ``i`` and row ``b``: the E4M3 scales of CSR
  blocks ``o_i // 16 + b`` and ``+ b + 1``, ``o_i`` the CSR position of the
  lane's first edge), and bits 28..31 of the lane's ``task_rows`` word hold
  ``o_i % 16``, so the kernel applies the scale of each edge's ORIGINAL
  16-edge block (``precision.py:52-73`` blocks the destination-major CSR).

Edge order inside a row piece is the CSR order, so a row's sum is a sequential
dot product per (row, block) followed by a sum over blocks in block order; the
column blocks depend only on the gathered length, so a row-sharded graph gives
bit-identical sums.  The builder runs on the weights' device with PyTorch ops;
it is cached by the runtime per ``weight_version``.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

import torch

from . import native

LANES = 32
CHUNK = 4                     # slots of one lane per chunk (the narrow width)
WIDE_CHUNK = 8                # the wide width: one 16-byte column load per lane
# A layout whose row pieces average at least this many edges uses wide chunks:
# half the loads, tags and ring steps per edge, for ~3.5 slots of padding per
# piece instead of ~1.5.  Measured (fp32, us per tick, 4 -> 8 slots): 166k /
# 25M 35.4 -> 32.0 (fp16 28.9 -> 24.2, fp8 29.8 -> 23.3, NVFP4 33.0 -> 27.6),
# 166k / 10M 18.2 -> 17.2, one rank of the 1.33M / 200M graph on 8 GPUs (6.5
# edges per piece) 56.5 -> 53.4, that graph on one GPU 478 -> 451.
WIDE_CHUNK_MIN_EDGES = 4
# E4M3 / NVFP4 layouts whose pieces average at least this many edges use
# 16-slot chunks (their weights are 1 / 0.5 bytes, so the extra padding costs
# little; fp16 would spill registers at that width).  166k / 25M (50-edge
# pieces): NVFP4 27.6 -> 26.0 us per tick, fp8 23.4 -> 23.3; 166k / 10M
# (20-edge pieces, 30 % padding at 16 slots): 21.5 -> 21.7, 18.1 -> 18.8.
WIDEST_CHUNK = 16
WIDEST_CHUNK_MIN_EDGES = 32
MAX_BLOCK_COLS = 65504        # 16-bit block-relative columns, block_cols = padding
MAX_ROWS = (1 << 28) - 1      # 28-bit rows in task_rows; ROW_NONE marks a padding lane
ROW_NONE = MAX_ROWS
WARPS = 31                    # consumer warps of a CTA
# Split length of sub-tasks in edges (a multiple of both chunk widths), by
# weight format (0: tasks are not split).  Splitting shortens the tail of a
# tick but adds row-sum planes that the update reads; measured at 166k / 25M it
# pays off for fp32 (8-slot chunks, 2,000 ticks: splits of 16 / 24 / 32 / 40 /
# 48 / 64 edges 47.5 / 36.6 / 31.0 / 31.9 / 32.1 / 32.7 us) and, with 4-slot
# chunks, costs the narrower formats (fp16 32.1 vs 30.5 us, NVFP4 38.5 vs
# 33.8 us).  A constant length cuts every row at the same edges whatever rows
# or chunk width a layout has, so sharded sums stay bit-identical.
SPLIT_EDGES = {native.F32: 32, native.F16: 0, native.E4M3: 0, native.NVFP4: 0}
MAX_PLANES = 32               # cap on blocks x splits (only degree-skewed graphs reach it)
# Slots per lane a task of several 32-piece segments holds at most (unsplit
# layouts; split layouts merge up to one split).  Layouts of short pieces
# otherwise hand out one task per ~2 chunks.  Measured on one rank's share of
# the 1.33M / 200M graph (166k rows x 1.33M columns, 23 blocks, 1-4 chunk
# pieces of 4 slots): 74.3 us per tick unmerged, 56.0 / 54.9 / 54.6 / 54.9 us
# with tasks of up to 24 / 28 / 32 / 40 slots per lane.
MERGE_SLOTS = 32
MAX_SEGMENT_CHUNKS = 63       # 6-bit segment length in a task's third word


def _u16(values: torch.Tensor) -> torch.Tensor:
    """Integers in [0, 65535] as the bit patterns of an int16 tensor (uint16 storage)."""
    values = values.to(torch.int32)
    return torch.where(values >= 32768, values - 65536, values).to(torch.int16)


def _i32(values: torch.Tensor) -> torch.Tensor:
    """Integers in [0, 2^32) as the bit patterns of an int32 tensor."""
    values = values.to(torch.int64)
    return torch.where(values >= 2**31, values - 2**32, values).to(torch.int32)


@dataclass
class TiledLayout:
    neurons: int          # destination rows of this layout
    n_edges: int
    ctas: int
    blocks: int
    block_cols: int
    buffers: int
    format: int
    stage_ptr: torch.Tensor    # int32 [ctas+1]: stages of CTA c
    stage_block: torch.Tensor  # int32 [stages]: column block of each stage
    task_ptr: torch.Tensor     # int32 [ctas+1]: tasks of CTA c
    # int32 [T, 4]: first slot, chunks, stage | split << 16 | segment chunks << 26
    # (0: one segment), then fp32: first row group, NVFP4: first scale pair
    tasks: torch.Tensor
    # int32, row ROW_NONE: padding lane.  fp32 [groups, 32]: segment k of task
    # q takes row group tasks[q, 3] + k; else [T, 32]: row (NVFP4: | phase << 28)
    task_rows: torch.Tensor
    col: torch.Tensor          # int16 storage of uint16 [S]
    weight: torch.Tensor       # [S] in the storage format (NVFP4: uint8 [S/2])
    scale_pairs: torch.Tensor | None  # int16 storage of uint16 (NVFP4)
    global_scale: torch.Tensor | None
    cols: int = 0         # length of the gathered source vector (0: same as neurons)
    splits: int = 1       # sub-task planes per block
    split_chunks: int = 1 << 20  # chunks of one sub-task
    chunk: int = CHUNK    # slots of one lane per chunk (4 or 8)
    _workspace: torch.Tensor | None = field(default=None, repr=False)

    def __post_init__(self) -> None:
        if self.cols == 0:
            self.cols = self.neurons

    def workspace(self) -> torch.Tensor:
        """The layout's device workspace (zero-filled on first use; calls keep it zeroed)."""
        if self._workspace is None:
            self._workspace = torch.zeros(self.workspace_bytes(), dtype=torch.uint8,
                                          device=self.col.device)
        return self._workspace

    @property
    def n_tasks(self) -> int:
        return self.tasks.shape[0]

    @property
    def n_stages(self) -> int:
        return self.stage_block.numel()

    @property
    def n_slots(self) -> int:
        return self.col.numel()

    @property
    def padding_fraction(self) -> float:
        return 1.0 - self.n_edges / max(self.n_slots, 1)

    def stream_bytes(self) -> int:
        """Bytes one tick streams from this layout (indices, weights, task tables)."""
        tables = sum(t.numel() * t.element_size() for t in (
            self.stage_ptr, self.stage_block, self.task_ptr, self.tasks, self.task_rows))
        if self.scale_pairs is not None:
            tables += self.scale_pairs.numel() * 2
        return self.col.numel() * 2 + self.weight.numel() * self.weight.element_size() + tables

    def workspace_bytes(self) -> int:
        """Device workspace one launch needs (barrier words + per-block row sums)."""
        return 256 + self.blocks * self.splits * self.neurons * 4

    def c_struct(self) -> "native._TiledLayout":
        def ptr(t):
            return t.data_ptr() if t is not None and t.numel() else None
        return native._TiledLayout(
            self.ctas, self.blocks, self.block_cols, self.buffers, self.format, self.splits,
            self.split_chunks, self.chunk, self.n_stages, self.n_tasks, self.n_slots,
            self.scale_pairs.numel() if self.scale_pairs is not None else 0,
            self.neurons, self.cols,
            ptr(self.stage_ptr), ptr(self.stage_block), ptr(self.task_ptr), ptr(self.tasks),
            ptr(self.task_rows), ptr(self.col), ptr(self.weight), ptr(self.scale_pairs),
            ptr(self.global_scale))


def plan_blocks(cols: int, ctas: int, smem_limit: int, smem_bytes) -> tuple[int, int, int]:
    """(blocks, block_cols, buffers) that fit one CTA's shared memory.

    Blocks are as large as one buffer allows when every CTA can hold a single
    block; with more blocks than CTAs, two half-size buffers pipeline a CTA's
    stages.
    """
    def cap(buffers: int) -> int:
        per_buffer = (smem_limit - smem_bytes(0, buffers)) // (4 * buffers) - 4
        return (min(per_buffer, MAX_BLOCK_COLS) // LANES) * LANES

    for buffers in (1, 2):
        width = cap(buffers)
        if width < LANES:
            raise ValueError("shared memory too small for a tiled layout")
        blocks = -(-cols // width)
        if blocks <= ctas or buffers == 2:
            block_cols = -(-(-(-cols // blocks)) // LANES) * LANES
            return blocks, block_cols, buffers
    raise AssertionError("unreachable")


def _apportion(weights: torch.Tensor, total: int) -> torch.Tensor:
    """Integer shares >= 1 of ``total`` proportional to ``weights`` (largest remainder)."""
    k = weights.numel()
    w = weights.double().clamp(min=1e-9)
    extra = total - k
    raw = w / w.sum() * extra
    share = raw.floor().long()
    left = extra - int(share.sum())
    if left > 0:
        share[torch.argsort(raw - share, descending=True, stable=True)[:left]] += 1
    return share + 1


def _stages(piece_len: torch.Tensor, ctas: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """(stage_cta, stage_block, stage_of_piece [n, blocks]) with stages sorted by CTA."""
    n, blocks = piece_len.shape
    device = piece_len.device
    if blocks > ctas:
        stage_block = torch.argsort(torch.arange(blocks, device=device) % ctas, stable=True)
        stage_cta = stage_block % ctas
        stage_of_block = torch.empty_like(stage_block)
        stage_of_block[stage_block] = torch.arange(blocks, device=device)
        return stage_cta, stage_block, stage_of_block.expand(n, blocks)
    cost = piece_len.long() + 1                      # edges + a row's own overhead
    share = _apportion(cost.sum(0), ctas)
    first = torch.cumsum(share, 0) - share
    stage_of = torch.empty((n, blocks), dtype=torch.int64, device=device)
    for k in range(blocks):
        before = torch.cumsum(cost[:, k], 0) - cost[:, k]   # cost of the rows above row r
        r = int(share[k])
        cuts = torch.arange(1, r, device=device) * int(cost[:, k].sum()) // r
        stage_of[:, k] = int(first[k]) + torch.searchsorted(cuts, before, right=True)
    stage_block = torch.repeat_interleave(torch.arange(blocks, device=device), share)
    stage_cta = torch.arange(ctas, device=device)
    return stage_cta, stage_block, stage_of


def split_length(fmt: int, edges: int, rows: int, blocks: int, longest: int) -> int:
    """Sub-task split length in edges for a graph (0: pieces are not split).

    ``longest`` is the longest row piece in edges.  Splitting only pays when a
    mean row piece (edges per (row, block)) is longer than one split (166k /
    25M fp32: 50 edges per piece, 36.9 vs 38.8 us with splits of 36 edges;
    166k / 10M: 20 edges, 19.2 unsplit vs 19.7 us); a degree-skewed graph gets
    longer splits so that blocks x splits stays within MAX_PLANES.  Always a
    multiple of WIDE_CHUNK, so both chunk widths cut a piece at the same edges.
    """
    split = SPLIT_EDGES.get(fmt, 0)
    if split > 0 and edges < split * rows * blocks:
        split = 0
    if split > 0 and blocks * -(-longest // split) > MAX_PLANES:
        split = -(-longest // max(1, MAX_PLANES // blocks))
        split = -(-split // WIDE_CHUNK) * WIDE_CHUNK
    return split


def chunk_width(edges: int, pieces: int, fmt: int = native.F32) -> int:
    """Slots per lane per chunk for a layout with ``pieces`` non-empty row pieces."""
    if fmt in (native.E4M3, native.NVFP4) and edges >= WIDEST_CHUNK_MIN_EDGES * max(pieces, 1):
        return WIDEST_CHUNK
    return WIDE_CHUNK if edges >= WIDE_CHUNK_MIN_EDGES * max(pieces, 1) else CHUNK


def graph_split(in_rowptr: torch.Tensor, in_col: torch.Tensor, fmt: int, *, neurons: int,
                cols: int, ctas: int, smem_limit: int, smem_bytes=None) -> int:
    """:func:`split_length` of a whole graph, for the layouts of its row blocks.

    A split cuts every row piece at the same edges, so row blocks laid out with
    the whole graph's split length sum every row as the whole graph's layout
    does (bit-identical sharded states), however their rows differ in degree.
    """
    if smem_bytes is None:
        lib = native.load_library()
        smem_bytes = lambda c, bufs: int(lib.nsb_tiled_smem_bytes(c, bufs))  # noqa: E731
    blocks, block_cols, _ = plan_blocks(cols, ctas, smem_limit, smem_bytes)
    rowptr = in_rowptr.to(torch.int64)
    edges = int(rowptr[-1])
    if edges == 0:
        return 0
    degree = rowptr[1:] - rowptr[:-1]
    rows = torch.repeat_interleave(torch.arange(neurons, dtype=torch.int32,
                                                device=in_col.device), degree)
    piece = rows * blocks + (in_col // block_cols).to(torch.int32)
    longest = int(torch.bincount(piece, minlength=neurons * blocks).max())
    return split_length(fmt, edges, neurons, blocks, longest)


def build_tiled_layout(in_rowptr: torch.Tensor, in_col: torch.Tensor, weight: torch.Tensor,
                       *, neurons: int, ctas: int, smem_limit: int, block_scales=None,
                       global_scale=None, smem_bytes=None, cols: int | None = None,
                       scale_offset: int = 0, split: int | None = None,
                       chunk: int | None = None) -> TiledLayout:
    """Build the tiled layout of one graph.

    ``weight`` is the CSR value array in its storage format (float32 / float16 /
    uint8 E4M3 codes / uint8 packed NVFP4).  ``neurons`` is the number of
    destination rows (``in_rowptr`` has neurons + 1 entries, starting at 0);
    ``cols`` is the length of the gathered source (default: ``neurons``).  For a
    block of rows cut out of a larger NVFP4 CSR, ``scale_offset`` is the CSR
    position of the block's first edge (it selects the original block scales,
    ``block_scales`` being those of the whole CSR).  ``ctas`` must not exceed
    the device's SM count (the kernel is a cooperative launch).
    """
    device = in_col.device
    if smem_bytes is None:
        lib = native.load_library()
        smem_bytes = lambda cols, bufs: int(lib.nsb_tiled_smem_bytes(cols, bufs))  # noqa: E731
    n, m = neurons, in_col.numel()
    cols = n if cols is None else cols
    if n > MAX_ROWS - 1:
        raise ValueError("too many rows for the tiled layout")
    if block_scales is not None:
        fmt = native.NVFP4
    elif weight.dtype == torch.uint8:
        fmt = native.E4M3
    elif weight.dtype == torch.float16:
        fmt = native.F16
    else:
        fmt = native.F32
    blocks, block_cols, buffers = plan_blocks(cols, ctas, smem_limit, smem_bytes)

    arange = lambda k: torch.arange(k, device=device)  # noqa: E731
    rowptr = in_rowptr.to(torch.int64)
    degree = rowptr[1:] - rowptr[:-1]
    row_of_edge = torch.repeat_interleave(arange(n), degree)
    col64 = in_col.to(torch.int64)
    block_of_edge = col64 // block_cols
    piece = row_of_edge * blocks + block_of_edge                       # (row, block) pair id
    piece_len = torch.bincount(piece, minlength=n * blocks).view(n, blocks)
    piece_start = (rowptr[:-1, None] + torch.cumsum(piece_len, 1) - piece_len).flatten()

    stage_cta, stage_block, stage_of = _stages(piece_len, ctas)
    n_stages = stage_block.numel()
    stage_ptr = torch.zeros(ctas + 1, dtype=torch.int64, device=device)
    torch.cumsum(torch.bincount(stage_cta, minlength=ctas), 0, out=stage_ptr[1:])

    # Non-empty pieces sorted by stage, then by chunk count (longest first),
    # then by row.  A task's chunk count is that of its first piece, as with a
    # sort by length, but its 32 rows ascend, so the warp's stores of their
    # sums into the row-sum plane touch a few lines instead of 32 (166k rows x
    # 1.33M columns, pieces of ~6.5 edges: 3.8M scattered stores a tick).
    group = stage_of.flatten()
    lengths = piece_len.flatten()
    order = torch.nonzero(lengths).flatten()
    K = chunk if chunk is not None else chunk_width(m, order.numel(), fmt)
    if K not in (CHUNK, WIDE_CHUNK, WIDEST_CHUNK) or (
            K == WIDEST_CHUNK and fmt not in (native.E4M3, native.NVFP4)):
        raise ValueError("chunk must be 4 or 8 (16 for E4M3 / NVFP4 weights)")
    K_SLOTS = LANES * K
    order = order[torch.sort(-((lengths[order] + K - 1) // K), stable=True).indices]
    order = order[torch.sort(group[order], stable=True).indices]
    sorted_group = group[order]
    group_size = torch.bincount(sorted_group, minlength=n_stages)
    group_start = torch.cumsum(group_size, 0) - group_size
    position = arange(order.numel()) - group_start[sorted_group]
    tasks_per_stage = (group_size + LANES - 1) // LANES
    stage_task = torch.cumsum(tasks_per_stage, 0) - tasks_per_stage
    pair_task = stage_task[sorted_group] + position // LANES
    pair_lane = position % LANES
    n_tasks = int(tasks_per_stage.sum())
    task_ptr = torch.zeros(ctas + 1, dtype=torch.int64, device=device)
    tasks_per_cta = torch.zeros(ctas, dtype=torch.int64, device=device)
    tasks_per_cta.index_add_(0, stage_cta, tasks_per_stage)
    torch.cumsum(tasks_per_cta, 0, out=task_ptr[1:])
    task_len = torch.zeros(n_tasks, dtype=torch.int64, device=device)
    task_len.scatter_reduce_(0, pair_task, lengths[order], reduce="amax")
    task_chunks = (task_len + K - 1) // K
    task_first = torch.cumsum(task_chunks * K_SLOTS, 0) - task_chunks * K_SLOTS
    slots = int((task_chunks * K_SLOTS).sum())
    if slots >= 2**31:
        raise ValueError("tiled layout exceeds 2^31 slots")
    task_stage = torch.repeat_interleave(arange(n_stages), tasks_per_stage)
    task_stage_local = task_stage - stage_ptr[stage_cta[task_stage]]
    pair_row = order // blocks

    # Slot of every edge: its pair's task and lane, and its rank inside the piece.
    rank_of_pair = torch.full((n * blocks,), -1, dtype=torch.int64, device=device)
    rank_of_pair[order] = arange(order.numel())
    r = rank_of_pair[piece]
    within = arange(m) - piece_start[piece]
    slot = (task_first[pair_task[r]] + (within // K) * K_SLOTS + pair_lane[r] * K
            + within % K)
    col = torch.full((slots,), block_cols, dtype=torch.int64, device=device)
    col[slot] = col64 - block_of_edge * block_cols

    task_rows = torch.full((n_tasks, LANES), ROW_NONE, dtype=torch.int64, device=device)
    scale_first = torch.zeros(n_tasks, dtype=torch.int64, device=device)
    scale_pairs = None
    if fmt == native.NVFP4:
        orig = piece_start[order] + scale_offset          # CSR position of each piece's first edge
        task_rows[pair_task, pair_lane] = pair_row | ((orig % 16) << 28)
        nibbles = torch.stack((weight & 15, weight >> 4), dim=1).flatten()[:m]
        codes = torch.zeros(slots, dtype=torch.uint8, device=device)
        codes[slot] = nibbles
        tiled_weight = (codes[0::2] | (codes[1::2] << 4)).contiguous()
        # Chunk c of a lane with phase p reads pair row (p + 4c) // 16 <= (11 + 4C) // 16.
        table_rows = ((15 - K + K * task_chunks) >> 4) + 1
        entries = table_rows * LANES
        scale_first = torch.cumsum(entries, 0) - entries
        n_pairs = int(entries.sum())
        # Blocks past a lane's last edge (its padding slots) get scale 0, so a
        # padding code (+0) never meets a neighbouring block's NaN scale.
        base = torch.zeros((n_tasks, LANES), dtype=torch.int64, device=device)
        base[pair_task, pair_lane] = orig // 16
        final = torch.full((n_tasks, LANES), -1, dtype=torch.int64, device=device)
        final[pair_task, pair_lane] = (orig + lengths[order] - 1) // 16
        task_of_entry = torch.repeat_interleave(arange(n_tasks), entries)
        local = arange(n_pairs) - scale_first[task_of_entry]
        lane_of_entry = local % LANES
        block = base[task_of_entry, lane_of_entry] + local // LANES
        final_of_entry = final[task_of_entry, lane_of_entry]
        last = block_scales.numel() - 1
        lo = torch.where(block <= final_of_entry, block_scales[block.clamp(max=last)], 0)
        hi = torch.where(block + 1 <= final_of_entry, block_scales[(block + 1).clamp(max=last)], 0)
        scale_pairs = _u16(lo.to(torch.int32) | (hi.to(torch.int32) << 8))
    else:
        task_rows[pair_task, pair_lane] = pair_row
        tiled_weight = torch.zeros(slots, dtype=weight.dtype, device=device)
        tiled_weight[slot] = weight
    # Sub-tasks: chunks [h * split, (h + 1) * split) of a task.  The split
    # length is this graph's (split_length), or the one given: row blocks of a
    # sharded graph take the whole graph's (graph_split).
    if split is None:
        split = split_length(fmt, m, n, blocks, int(task_len.max()) if n_tasks else 1)
    longest = int(task_chunks.max()) if n_tasks else 1   # in chunks from here on
    split = split // K if split > 0 else 1 << 30
    split = max(1, min(split, 1 << 30))
    splits = max(1, -(-longest // split))
    unsplit = splits == 1
    split = min(split, max(longest, 1))
    # Tasks: runs of consecutive groups of one stage with one chunk count c are
    # merged, up to MERGE_SLOTS slots per lane (and one split) per task, into tasks
    # of several segments (c chunks each, one group's 32 pieces per segment),
    # so layouts of short pieces do not hand out a task per 32 pieces.  Only
    # fp32: the narrower formats keep one group per task (NVFP4's task carries
    # the group's scale table).  Merging moves no slot: a task's groups are
    # consecutive in slot order.
    group_chunks = task_chunks
    if fmt == native.F32 and n_tasks:
        target = MERGE_SLOTS // K if unsplit else min(split, MERGE_SLOTS // K)
        run_head = torch.ones(n_tasks, dtype=torch.bool, device=device)
        run_head[1:] = (task_stage[1:] != task_stage[:-1]) | (group_chunks[1:] != group_chunks[:-1])
        run_first = torch.nonzero(run_head).flatten()
        position = arange(n_tasks) - run_first[torch.cumsum(run_head.long(), 0) - 1]
        per_task = torch.where(group_chunks <= MAX_SEGMENT_CHUNKS,
                               torch.clamp(target // group_chunks.clamp(min=1), min=1), 1)
        head = position % per_task == 0
        first_group = torch.nonzero(head).flatten()
        groups = torch.bincount(torch.cumsum(head.long(), 0) - 1)
        merged_chunks = group_chunks[first_group] * groups
        segment = torch.where(groups > 1, group_chunks[first_group], 0)
        merged_word = first_group                       # the task's first row group
    else:
        first_group = arange(n_tasks)
        merged_chunks = group_chunks
        segment = torch.zeros_like(group_chunks)
        merged_word = scale_first                       # NVFP4: the task's scale table
    n_merged = first_group.numel()
    if unsplit and n_merged:
        split = max(split, int(merged_chunks.max()))   # one sub-task per task
    n_sub = (merged_chunks + split - 1) // split
    sub_task = torch.repeat_interleave(arange(n_merged), n_sub)
    sub_h = arange(sub_task.numel()) - (torch.cumsum(n_sub, 0) - n_sub)[sub_task]
    sub_chunks = torch.clamp(merged_chunks[sub_task] - sub_h * split, max=split)
    # Within a stage: longest sub-tasks first (tasks keep their order otherwise).
    sub_group = first_group[sub_task]
    sub_stage = task_stage[sub_group]
    sub_order = torch.sort(-sub_chunks, stable=True).indices
    sub_order = sub_order[torch.sort(sub_stage[sub_order], stable=True).indices]
    sub_task, sub_h, sub_chunks = sub_task[sub_order], sub_h[sub_order], sub_chunks[sub_order]
    sub_group = first_group[sub_task]
    tasks = torch.stack((task_first[sub_group] + sub_h * split * K_SLOTS, sub_chunks,
                         task_stage_local[sub_group] | (sub_h << 16) | (segment[sub_task] << 26),
                         merged_word[sub_task]), dim=1)
    subs_per_cta = torch.zeros(ctas, dtype=torch.int64, device=device)
    subs_per_cta.index_add_(0, stage_cta[task_stage[sub_group]], torch.ones_like(sub_group))
    torch.cumsum(subs_per_cta, 0, out=task_ptr[1:])
    if fmt != native.F32:
        task_rows = task_rows[sub_group]               # one row word per lane of each task
    return TiledLayout(
        neurons=n, n_edges=m, ctas=ctas, blocks=blocks, block_cols=block_cols, buffers=buffers,
        format=fmt, stage_ptr=stage_ptr.to(torch.int32), stage_block=stage_block.to(torch.int32),
        task_ptr=task_ptr.to(torch.int32), tasks=tasks.to(torch.int32).contiguous(),
        task_rows=_i32(task_rows).contiguous(), col=_u16(col), weight=tiled_weight,
        scale_pairs=scale_pairs, global_scale=global_scale, cols=cols, splits=splits,
        split_chunks=split, chunk=K)


def emulate(layout: TiledLayout, source: torch.Tensor) -> torch.Tensor:
    """What the kernel computes, j = W @ source (B = 1), in float64 on any device.

    Every slot is decoded the way the kernel decodes it (including the NVFP4
    scale-pair lookup); used by the tests to check a layout without a GPU.
    """
    x = source.reshape(-1).double()
    dev = x.device
    out = torch.zeros(layout.neurons, dtype=torch.float64, device=dev)
    if layout.n_slots == 0:
        return out
    slots = torch.arange(layout.n_slots, device=dev)
    first = layout.tasks[:, 0].long()
    by_slot = torch.argsort(first)           # (sub-)tasks are not stored in slot order
    task = by_slot[torch.searchsorted(first[by_slot], slots, right=True) - 1]
    local = slots - first[task]
    K = layout.chunk
    chunk, lane, e = local // (LANES * K), (local % (LANES * K)) // K, local % K
    third = layout.tasks[:, 2].long()
    if layout.format != native.F32:
        word = layout.task_rows.long()[task, lane] & 0xFFFFFFFF
    else:
        segment = (third >> 26) & 63
        length = torch.where(segment > 0, segment, layout.tasks[:, 1].long())[task]
        group = layout.tasks[:, 3].long()[task] + chunk // length
        word = layout.task_rows.long()[group, lane] & 0xFFFFFFFF
        chunk = chunk % length
    col = layout.col.long() & 0xFFFF
    cta = torch.searchsorted(layout.task_ptr.long(), torch.arange(layout.n_tasks, device=dev),
                             right=True) - 1
    stage = layout.stage_ptr.long()[cta] + (third & 0xFFFF)
    block = layout.stage_block.long()[stage][task]
    chunk = chunk + ((third >> 16) & 0x3FF)[task] * layout.split_chunks
    padded = torch.cat([x, torch.zeros(layout.blocks * layout.block_cols + 1 - x.numel(),
                                       dtype=x.dtype, device=dev)])
    gathered = torch.where(col == layout.block_cols, torch.zeros_like(x[:1]),
                           padded[block * layout.block_cols + col.clamp(max=layout.block_cols - 1)])
    value = _decoded_slots(layout, task, chunk, lane, e, word).double() * gathered
    row = word & MAX_ROWS
    keep = row != ROW_NONE
    out.index_add_(0, row[keep], value[keep])
    return out


def _decoded_slots(layout: TiledLayout, task, chunk, lane, e, word) -> torch.Tensor:
    if layout.format == native.F32 or layout.format == native.F16:
        return layout.weight.float()
    from .precision import e2m1_to_float, e4m3_to_float
    g = layout.global_scale.float()
    if layout.format == native.E4M3:
        return e4m3_to_float(layout.weight) * g
    codes = torch.stack((layout.weight & 15, layout.weight >> 4), dim=1).flatten()
    p = (word >> 28) + layout.chunk * chunk
    entry = layout.tasks[:, 3].long()[task] + (p >> 4) * LANES + lane
    pair = layout.scale_pairs.long()[entry] & 0xFFFF
    scale = torch.where((p & 15) + e >= 16, pair >> 8, pair & 0xFF).to(torch.uint8)
    return e2m1_to_float(codes) * (e4m3_to_float(scale) * g)


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


ROLLOUT_CAP = 32  # longest launch of a streamed rollout on the tiled path


def rollout_chunks(ticks: int, cap: int = ROLLOUT_CAP, first: int = 2) -> list[int]:
    """Launch lengths of a streamed rollout of ``ticks`` ticks: a head of
    ``first``, 2 * ``first``, ... (doubling while the head and its mirror fit
    and below ``cap``), the rest of the ticks in near-equal launches of at
    most ``cap``, then the head in reverse.  The upload before the first
    launch and the download after the last one are short, and along the head
    each launch's drives (twice as many ticks) upload while the launch before
    it runs.  The middle launches are not bounded by the last head launch
    (20 ticks from 1: 1-2-4-6-4-2-1; 13: 1-2-7-2-1)."""
    head, size = [], first
    while size < cap and 2 * (sum(head) + size) <= ticks:
        head.append(size)
        size *= 2
    middle = ticks - 2 * sum(head)
    pieces = -(-middle // cap)  # the middle in near-equal launches of at most `cap`
    body = [middle // pieces + (i < middle % pieces) for i in range(pieces)] if pieces else []
    return head + body + head[::-1]
