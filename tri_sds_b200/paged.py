"""Paged KV memory in SGLang's layout.

SGLang keeps a model's KV cache in per-layer token pools
(``token_to_kv_pool.k_buffer[layer]`` / ``v_buffer[layer]``, each
``[pool_rows, Hkv, D]``) and maps request positions to pool rows through
``req_to_token_pool.req_to_token`` (int32 ``[max_reqs, max_context]``); a
batch names its requests' table rows with ``req_pool_indices``.  The
reference worker receives SGLang's ScheduleBatch (tri_sds/worker.py:3-4,
59-61), whose requests own exactly this memory.

``PagedKV`` holds those tensors for one model.  ``QwenModel(kv=PagedKV(...))``
then writes and reads its K/V through them (tsds_qk_norm_rope_kv_paged,
tsds_verify_attention_paged) instead of its own contiguous cache, and the
EAGLE engine commits an accepted tree by rewriting table entries
(tsds_tree_commit_paged) instead of moving K/V rows.  ``PagedKV.wrap`` takes
SGLang's own tensors; ``PagedKV.allocate`` builds an engine-owned pool with a
scattered table (rows handed out in random order, as a long-running
allocator leaves them) for standalone use and tests.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass
class PagedKV:
    k_pools: list            # per layer [pool_rows, Hkv, D] bf16
    v_pools: list
    table: torch.Tensor      # int32 [reqs, table_ld]: pool row of each request position
    req_rows: torch.Tensor | None = None   # int64 [B]: the batch's table rows (None: row b)
    page_size: int = 1       # a multiple of 64: every aligned 64 positions are 64 consecutive pool rows

    def __post_init__(self):
        assert len(self.k_pools) == len(self.v_pools) and self.k_pools
        k0 = self.k_pools[0]
        for k, v in zip(self.k_pools, self.v_pools):
            assert k.shape == k0.shape and v.shape == k0.shape and k.dtype == torch.bfloat16
            assert k.is_contiguous() and v.is_contiguous()
        assert self.table.dtype == torch.int32 and self.table.dim() == 2 and self.table.is_contiguous()
        if self.req_rows is not None:
            assert self.req_rows.dtype == torch.int64

    @property
    def pool_rows(self) -> int:
        return int(self.k_pools[0].shape[0])

    @property
    def n_kv_heads(self) -> int:
        return int(self.k_pools[0].shape[1])

    @property
    def table_ld(self) -> int:
        return int(self.table.shape[1])

    @classmethod
    def wrap(cls, k_buffer, v_buffer, req_to_token, req_pool_indices=None, page_size: int = 1) -> "PagedKV":
        """SGLang's tensors as they are: token_to_kv_pool.k_buffer / v_buffer,
        req_to_token_pool.req_to_token and the batch's req_pool_indices."""
        rr = None if req_pool_indices is None else req_pool_indices.to(torch.int64).contiguous()
        return cls(list(k_buffer), list(v_buffer), req_to_token, rr, page_size)

    @classmethod
    def from_batch(cls, batch, page_size: int = 1) -> "PagedKV":
        """The KV memory a SGLang ScheduleBatch carries: its request-to-token
        table (``batch.req_to_token_pool.req_to_token``), its token pool's
        per-layer buffers (``batch.token_to_kv_pool_allocator.get_kvcache()``,
        or ``batch.token_to_kv_pool`` where a batch holds the pool itself) and
        its requests' table rows (``batch.req_pool_indices``)."""
        alloc = getattr(batch, "token_to_kv_pool_allocator", None)
        pool = alloc.get_kvcache() if alloc is not None else getattr(batch, "token_to_kv_pool", None)
        if pool is None or getattr(batch, "req_to_token_pool", None) is None:
            raise ValueError("the batch carries no token pool / request-to-token table")
        return cls.wrap(pool.k_buffer, pool.v_buffer, batch.req_to_token_pool.req_to_token,
                        getattr(batch, "req_pool_indices", None), page_size)

    @classmethod
    def allocate(cls, n_layers: int, batch: int, max_seq: int, n_kv_heads: int, head_dim: int, device,
                 page_size: int = 1, seed: int = 0, spare: int = 16) -> "PagedKV":
        """Engine-owned pools for `batch` sequences of up to `max_seq`
        positions: every position gets its own pool row (page_size 1) or every
        64-position page its own page of rows, handed out in a random order;
        the table's rows are taken in a random order too."""
        assert page_size == 1 or page_size % 64 == 0
        g = torch.Generator().manual_seed(seed)
        if page_size == 1:
            pool_rows = batch * max_seq + spare
            rows = torch.randperm(pool_rows, generator=g)[:batch * max_seq].reshape(batch, max_seq)
        else:
            npg = -(-max_seq // page_size)
            pages = torch.randperm(batch * npg + spare, generator=g)[:batch * npg].reshape(batch, npg)
            rows = (pages.unsqueeze(-1) * page_size + torch.arange(page_size)).reshape(batch, -1)[:, :max_seq]
            pool_rows = (batch * npg + spare) * page_size
        reqs = batch + spare
        req = torch.randperm(reqs, generator=g)[:batch]
        table = torch.zeros(reqs, max_seq, dtype=torch.int32)
        table[req] = rows.to(torch.int32)
        dev = torch.device(device)
        pools = [torch.zeros(pool_rows, n_kv_heads, head_dim, dtype=torch.bfloat16, device=dev)
                 for _ in range(2 * n_layers)]
        return cls(pools[:n_layers], pools[n_layers:], table.to(dev), req.to(dev), page_size)

    def gather(self, layer: int, b: int, n: int):
        """(K, V) of the first n positions of sequence b at `layer`, [Hkv, n, D]
        (tests / inspection)."""
        req = b if self.req_rows is None else int(self.req_rows[b])
        rows = self.table[req, :n].long()
        return (self.k_pools[layer][rows].transpose(0, 1), self.v_pools[layer][rows].transpose(0, 1))
