"""SeoulKV4 sparse-decode attention for NVIDIA B200 (sm_100a).

Drop-in for the reference's Python operator API::

    from seoulkv_b200 import SeoulKV4, SeoulKV4Config, SeoulKV4Index
    index = SeoulKV4Index.build(k, v, sink=128, local=256, nprobe=384)
    with SeoulKV4(device="cuda:0", k=k, v=v, index=index) as attn:
        attn.run(q0)
        y = attn.run(q1).to_torch()
"""

from seoulkv_b200.api import SeoulKV4
from seoulkv_b200.batched import BatchResult, SeoulKV4Batch
from seoulkv_b200.config import SeoulKV4Config
from seoulkv_b200.index import SeoulKV4Index
from seoulkv_b200.result import DecodeResult

__all__ = ["BatchResult", "DecodeResult", "SeoulKV4", "SeoulKV4Batch", "SeoulKV4Config", "SeoulKV4Index"]
