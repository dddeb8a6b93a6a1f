"""Block-sparse attention masks (CPU): CSR tables, token masks, window covers, reference path."""
import pytest
import torch

from ditserve_b200 import ops
from ditserve_b200 import ops as A


def test_block_sparse_table_csr():
    m = torch.tensor([[1, 0, 1], [0, 1, 0]], dtype=torch.bool)
    off, idx = A.block_sparse_table(m)
    assert off.tolist() == [0, 2, 3] and idx.tolist() == [0, 2, 1]
    assert off.dtype == torch.int32 and idx.dtype == torch.int32
    with pytest.raises(ValueError):
        A.block_sparse_table(torch.tensor([[1, 0], [0, 0]], dtype=torch.bool))


def test_sliding_window_mask_covers_every_pair_in_the_window():
    sq, sk, w = 700, 900, 150
    bm = A.sliding_window_block_mask(sq, sk, w)
    assert bm.shape == (3, 8)
    tm = A.token_mask(bm, sq, sk)
    i = torch.arange(sq)[:, None]
    j = torch.arange(sk)[None, :]
    need = (i - j).abs() <= w
    assert bool(tm[need].all())
    assert bm.float().mean() < 1.0  # something was skipped


def test_tile_window_mask_covers_every_pair_in_the_3d_window():
    grid, win = (3, 12, 20), (1, 3, 4)
    bm = A.tile_window_block_mask(grid, win)
    n = grid[0] * grid[1] * grid[2]
    tm = A.token_mask(bm, n, n)
    idx = torch.arange(n)
    c = torch.stack([idx // (grid[1] * grid[2]), (idx // grid[2]) % grid[1], idx % grid[2]], 1)
    d = (c[:, None, :] - c[None, :, :]).abs()
    need = (d <= torch.tensor(win)).all(-1)
    assert bool(tm[need].all())


def test_reference_path_applies_the_block_mask():
    torch.manual_seed(0)
    B, S, H, D = 2, 600, 2, 64
    q = torch.randn(B, S, H * D)
    k = torch.randn(B, S, H * D)
    v = torch.randn(B, S, H * D)
    bm = A.sliding_window_block_mask(S, S, 100)
    o = ops.attention(q, k, v, H, block_mask=bm)
    # the same statement with the token mask spelled out per (query, key)
    tm = A.token_mask(bm, S, S)
    qh = q.view(B, S, H, D).transpose(1, 2)
    kh = k.view(B, S, H, D).transpose(1, 2)
    vh = v.view(B, S, H, D).transpose(1, 2)
    s = (qh @ kh.transpose(-1, -2)) / D ** 0.5
    s = s.masked_fill(~tm, float("-inf"))
    ref = (torch.softmax(s, -1) @ vh).transpose(1, 2).reshape(B, S, H * D)
    assert torch.allclose(o, ref, atol=1e-5, rtol=1e-5)
    dense = ops.attention(q, k, v, H)
    assert not torch.allclose(o, dense, atol=1e-3)
    with pytest.raises(ValueError):
        ops.attention(q.view(B * S, -1), k.view(B * S, -1), v.view(B * S, -1), H, block_mask=bm,
                      cu_seqlens_q=torch.tensor([0, S, 2 * S]), cu_seqlens_k=torch.tensor([0, S, 2 * S]))
