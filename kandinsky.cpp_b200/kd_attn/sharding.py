"""Head sharding of the CrossDiT attention across the GPUs of one box.

Heads are independent, so rank r of n owns heads [r*H/n, (r+1)*H/n): its inputs are the
matching column slice of the Q/K/V projections ([H/n*128, L, N]), its output the same slice
of the attention result.  kd_attn_allgather_heads gathers the slices rank-major with one
ncclAllGather ([n][N*L][H/n*128]) and permutes them into [N*L][H*128] rows (= [C, L, N]),
the layout the out-projection (crossdit.hpp:153) consumes.  The functions here state that
layout on the host (numpy / torch CPU), so the gather logic can be checked without GPUs.
"""
from __future__ import annotations


def head_range(rank: int, n_ranks: int, n_heads: int):
    """[first, last) heads owned by `rank`; n_heads must be a multiple of n_ranks."""
    if n_ranks <= 0 or n_heads % n_ranks:
        raise ValueError(f"{n_heads} heads do not split over {n_ranks} ranks")
    per = n_heads // n_ranks
    return rank * per, (rank + 1) * per


def column_shard(x, rank: int, n_ranks: int, n_heads: int, head_dim: int = 128):
    """The rank's columns of a (N, L, C) projection (ggml [C, L, N])."""
    h0, h1 = head_range(rank, n_ranks, n_heads)
    return x[..., h0 * head_dim:h1 * head_dim]


def unshard_rank_major(gathered, n_ranks: int):
    """(n_ranks, rows, shard_cols) rank-major all-gather result -> (rows, n_ranks*shard_cols).

    Host statement of what unshard_kernel (csrc/kd_kernels.cu) does after ncclAllGather.
    """
    R, rows, cols = gathered.shape
    if R != n_ranks:
        raise ValueError(f"expected {n_ranks} shards, got {R}")
    if hasattr(gathered, "permute"):  # torch tensor
        return gathered.permute(1, 0, 2).reshape(rows, R * cols)
    return gathered.transpose(1, 0, 2).reshape(rows, R * cols)  # numpy array
