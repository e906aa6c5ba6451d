"""mrl_b200 — B200 (sm_100a) PaxBlock64 bitplane scan behind the reference's scan interface.

The compute path is libmrl_b200.so (CUDA kernels + C ABI, include/mrl_cuda.h); this package is
its host-side mirror of the reference crate's scan API. Importing it loads the library and fails
loudly when it is absent.
"""
from ._capi import LIB_PATH, MrlError, load  # noqa: F401
from .api import (  # noqa: F401
    BLOCK_BYTES,
    DEFAULT_STRATUM4_WEIGHT,
    VECTORS_PER_BLOCK,
    Device,
    EdenFit,
    EngineConfig,
    MidCodec,
    PrefixCodec,
    QueryPipeline,
    QueryPlan,
    ScanConfig,
    ScanMode,
    ScoredHit,
    Segment,
    StrataDepth,
    VectorId,
    default_device,
    encode_blocks,
    row_id_to_vector_id,
    query_scan,
    QueryStream,
    MAX_INFLIGHT,
    scan_blocks,
    scan_blocks_batch,
    scan_blocks_stats,
    ScanStats,
    scored_hits_to_row_ids,
    vector_scores,
    score_bound,
    control_words,
)
from .index import (  # noqa: F401
    DeviceRing,
    IndexDir,
    PendingVector,
    SegmentError,
    SegmentWriter,
    config_from_json,
    config_to_json,
    id_map_from_pages,
    load_segment,
    rerank_exact_rows,
)
from .shard import (  # noqa: F401
    BatchShardExchange,
    PeerExchange,
    ShardExchange,
    merge_topk_host,
    pack_records,
    record_bytes,
    shard_range,
    unpack_records,
)

load()
