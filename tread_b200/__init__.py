"""tread_b200: B200-native (sm_100a) chunk-reuse hot path with tread's engine/store API.

    from tread_b200 import Engine, BlockStore
    eng = Engine(model, BlockStore(budget_bytes, cpu_budget_bytes))
    logits, cache, stats = eng.prefill(prefix_ids, docs, query_ids, ratio=0.2)

Several GPUs (one process per GPU, NCCL):
    tread_b200.tp.TPQwen2Rows   the model split by KV head; pass it to Engine in place of the model
    tread_b200.dp.ShardedEngine replicas with the block store sharded by content hash
"""
from tread_b200.engine import Engine, RequestStats, prefill_full
from tread_b200.store import Block, BlockStore, StoreStats, block_key

__all__ = ["Engine", "BlockStore", "Block", "StoreStats", "RequestStats", "block_key", "prefill_full"]
