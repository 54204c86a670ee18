"""1-bit candidate generation on the fp8 tensor cores, and the LiNR V3 cascade.

The reference scores 1-bit codes with popcounts: ``score = 64 W − 2 Σ_w
popcount(q_w ^ x_w)`` (retrieve/src/retrieve/ops/reference/oporp_1bit_match_topk.py:9-41),
the ``OneBitKNN`` stage of LiNR V3 (retrieve/src/retrieve/modules/linr.py:118-162).
For codes mapped to ±1 vectors that score is their dot product, so here the item
codes are expanded once, at registration, into a ±1 fp8 e4m3 table
(``bits_to_pm1(…, "e4m3")``, 8 bytes per 64 code bits) and every batch is one
``kind::f8f6f4`` tensor-core scan whose fp32 accumulator is the score: ±1 is
exact in e4m3 and every partial sum is an integer of at most 64 W in
magnitude, so the scores are exact — the same scores and the same (score
desc, id asc) ordering as the popcount path, at tensor-core rather than
POPC-pipe throughput. Widths with
64·W in {128, 256, 512} bits use the tensor cores; other widths use the exact
popcount kernel (``oporp_1bit_match_topk_full``).
"""

from __future__ import annotations

import torch
from torch import Tensor

from retrieve_b200 import ops

TENSOR_CORE_BITS = (128, 256, 512)


class PackedBitsIndex:
    """An item table of 1-bit codes ``[N, W]`` int64 (bit b of word w =
    coordinate 64 w + b) prepared for top-k by 1-bit match score."""

    def __init__(self, item_bits: Tensor) -> None:
        if item_bits.dim() != 2 or item_bits.dtype != torch.int64:
            raise ValueError("item_bits must be [N, W] int64")
        self.n, self.w = item_bits.shape
        self.tensor_cores = 64 * self.w in TENSOR_CORE_BITS
        if self.tensor_cores:
            self.table = ops.bits_to_pm1(item_bits, "e4m3")
            self.bits = None
        else:
            self.table = None
            self.bits = item_bits.contiguous()

    def topk(self, query_bits: Tensor, k: int, id_offset: int = 0) -> tuple[Tensor, Tensor]:
        """``(ids [B, k] int64, scores [B, k] fp32)``: the k best items by
        ``64 W − 2·hamming``, ties to the lower id; ``id_offset`` is added to
        the ids (row-sharded tables)."""
        if query_bits.dim() != 2 or query_bits.shape[1] != self.w:
            raise ValueError(f"query_bits must be [B, {self.w}] int64")
        if self.tensor_cores:
            from retrieve_b200 import _lib

            q = ops.bits_to_pm1(query_bits.contiguous(), "e4m3")
            return ops.scaled_topk(q, None, self.table, None, k, _lib.RB_E4M3, id_offset)
        ids, scores = ops.oporp_1bit_match_topk_full(query_bits, self.bits, min(k, self.n))
        if ids.shape[1] < k:  # fewer items than k: pad like the dense paths
            pad = k - ids.shape[1]
            ids = torch.cat([ids, ids.new_full((ids.shape[0], pad), -1)], dim=1)
            scores = torch.cat([scores, scores.new_full((scores.shape[0], pad), float("-inf"))], dim=1)
        if id_offset:
            ids = torch.where(ids >= 0, ids + id_offset, ids)
        return ids, scores


def onebit_rerank_topk(
    query: Tensor, query_bits: Tensor, bits_index: PackedBitsIndex, item_embs: Tensor, pool: int, k: int
) -> tuple[Tensor, Tensor]:
    """LiNR V3 without a filter (modules/linr.py:155-162): the 1-bit top-``pool``
    candidates, rescored exactly (fp32 dots of ``query`` and ``item_embs`` rows,
    ``fused_masked_knn_topk``) to the top ``k``. Pool slots past the corpus
    (id -1) are not scored."""
    if k > pool:
        raise ValueError(f"k={k} exceeds candidate_pool={pool}")
    cand, _ = bits_index.topk(query_bits, pool)
    counts = (cand >= 0).sum(dim=1)
    return ops.fused_masked_knn_topk(query, item_embs, cand, counts, k)
