"""Row-sharded multi-GPU quantization (one process per GPU, torch.distributed).

Blocks are independent once the global-scale multiplier is known, and the
multiplier only needs the tensor-wide |x| maximum, so the one exchange step is
a MAX all-reduce of a single float32 (NCCL over NVLink on GPUs; exact and
order-independent).  Each rank reads only its own rows.

Row ranges are handed out in whole 128-row tiles, so every rank but the last
owns a multiple of 128 rows.  Then each rank's swizzled scale slab
``[round_up(rows_r, 128), round_up(K/16, 4)]`` is exactly the matching slice
of the whole tensor's scale buffer, and concatenating the ranks' codes and
scales reproduces the single-GPU output byte for byte.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

TILE_ROWS = 128


def shard_rows(total_rows: int, world_size: int, rank: int) -> tuple[int, int]:
    """[start, stop) rows of ``rank``: whole 128-row tiles, remainder on the last ranks."""
    if world_size < 1 or not 0 <= rank < world_size:
        raise ValueError("bad rank / world size")
    tiles = -(-total_rows // TILE_ROWS)
    base, extra = divmod(tiles, world_size)
    # the first (world_size - extra) ranks get `base` tiles, the rest `base + 1`
    lo_ranks = world_size - extra
    start_tile = rank * base + max(0, rank - lo_ranks)
    n_tiles = base + (1 if rank >= lo_ranks else 0)
    start = min(start_tile * TILE_ROWS, total_rows)
    stop = min((start_tile + n_tiles) * TILE_ROWS, total_rows)
    return start, stop


def scale_slab_rows(start: int, stop: int) -> tuple[int, int]:
    """Rows of the whole tensor's swizzled scale buffer that a shard's slab covers."""
    return start, start + -(-(stop - start) // TILE_ROWS) * TILE_ROWS


def all_reduce_amax(amax: torch.Tensor, group=None) -> torch.Tensor:
    """In-place MAX all-reduce of the per-rank |x| maximum (float32 [1]).

    The reduction runs on the float's bit pattern as int32.  An |x| maximum is
    +0, a positive finite value, +inf or a NaN with the sign bit clear, and
    for those patterns signed-integer order is value order with NaN above
    +inf.  So the result is the largest amax, and a NaN on any rank wins, as
    ``x.abs().max()`` over the whole tensor would give.  A float MAX would
    not promise that: NCCL's and gloo's float maximum may drop a NaN operand.
    """
    if amax.dtype != torch.float32:
        raise ValueError("amax must be float32")
    if dist.is_available() and dist.is_initialized():
        bits = amax.view(torch.int32)
        dist.all_reduce(bits, op=dist.ReduceOp.MAX, group=group)
    return amax


def quantize_row_shard(x_local: torch.Tensor, fp8_max: float = 448.0, *, group=None,
                       backend: str = "scalesweep_mse", is_sf_swizzled_layout: bool = True,
                       output: torch.Tensor | None = None,
                       output_scale: torch.Tensor | None = None):
    """Quantize this rank's rows with the tensor-wide global scale.

    Returns ``(codes, scales, input_scale)``; ``input_scale`` is the device
    multiplier ``fp8_max*6 / amax_global`` shared by every rank.
    """
    from . import _quant, global_scale
    from .custom import create_fp4_output_tensors

    if x_local.dim() != 2:
        raise ValueError("x_local must be 2-D [rows, K]")
    dev = x_local.device
    if x_local.shape[0] > 0:
        amax = global_scale.absmax(x_local)
    else:
        amax = torch.zeros(1, dtype=torch.float32, device=dev)
    all_reduce_amax(amax, group)
    gsi = global_scale.global_scale_from_amax(amax, fp8_max)
    m, k = x_local.shape
    if output is None or output_scale is None:
        output, output_scale = create_fp4_output_tensors(m, k, dev, is_sf_swizzled_layout)
    kind = {"scalesweep_mse": "mse", "scalesweep_mse_reference": "reference",
            "scalesweep_mse128": "mse128", "rtn": "rtn"}[backend]
    _quant.launch(kind, x_local, gsi, is_sf_swizzled_layout, output, output_scale)
    return output, output_scale.view(torch.float8_e4m3fn), gsi
