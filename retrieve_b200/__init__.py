"""retrieve_b200: the scoring-and-selection hot path of torchretrieve
(rmnigm/retrieve) as hand-written sm_100a CUDA kernels.

``retrieve_b200.ops`` is the op namespace (``torch.ops.retrieve.*``), a drop-in
for ``retrieve.ops.triton``; ``retrieve_b200.shard`` row-shards a corpus over
several GPUs and merges the per-shard top-k after an NCCL all-gather. The
kernels live in ``libretrieve_b200.so`` (C-ABI: ``include/retrieve_b200.h``),
built in-tree by ``python -m retrieve_b200.build``.
"""

__version__ = "0.1.0"
