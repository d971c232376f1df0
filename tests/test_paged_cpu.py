"""Paged KV host side (no GPU): the engine-owned allocation's invariants and
the wrapping of SGLang's tensors as a ScheduleBatch carries them."""
from types import SimpleNamespace

import pytest
import torch

from tri_sds_b200.paged import PagedKV


@pytest.mark.parametrize("page", [1, 64])
def test_allocate_gives_every_position_its_own_row(page):
    kv = PagedKV.allocate(n_layers=2, batch=3, max_seq=200, n_kv_heads=2, head_dim=128, device="cpu",
                          page_size=page, seed=5)
    assert len(kv.k_pools) == 2 and kv.k_pools[0].shape == (kv.pool_rows, 2, 128)
    rows = kv.table[kv.req_rows].long()
    assert rows.shape == (3, 200)
    assert int(rows.min()) >= 0 and int(rows.max()) < kv.pool_rows
    assert rows.unique().numel() == rows.numel()          # no two positions share a pool row
    if page == 64:
        # every aligned run of 64 positions is 64 consecutive pool rows, starting on a page
        for b in range(3):
            for p0 in range(0, 200, 64):
                r = rows[b, p0:p0 + 64]
                assert int(r[0]) % 64 == 0 and torch.equal(r - r[0], torch.arange(r.numel()))
    else:
        assert not torch.equal(rows[0], torch.sort(rows[0]).values)   # scattered, not in order


def test_from_batch_wraps_sglangs_tensors():
    k = [torch.zeros(50, 2, 128, dtype=torch.bfloat16) for _ in range(3)]
    v = [torch.zeros(50, 2, 128, dtype=torch.bfloat16) for _ in range(3)]
    table = torch.zeros(4, 64, dtype=torch.int32)
    pool = SimpleNamespace(k_buffer=k, v_buffer=v)
    batch = SimpleNamespace(token_to_kv_pool_allocator=SimpleNamespace(get_kvcache=lambda: pool),
                            req_to_token_pool=SimpleNamespace(req_to_token=table),
                            req_pool_indices=torch.tensor([2, 0], dtype=torch.int32))
    kv = PagedKV.from_batch(batch)
    assert kv.k_pools[1] is k[1] and kv.table is table and kv.req_rows.dtype == torch.int64
    assert kv.req_rows.tolist() == [2, 0] and kv.pool_rows == 50 and kv.table_ld == 64
    with pytest.raises(ValueError):
        PagedKV.from_batch(SimpleNamespace(input_ids=None))
