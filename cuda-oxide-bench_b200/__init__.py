"""B200-native (sm_100a) gated delta-rule linear attention.

Entry points (all on CUDA tensors, all through the C ABI of libgdn_b200.so):

* :func:`gdn_decode` — one GDN decode step, state updated in place.
* :func:`kda_decode` — one KDA (per-channel gate) decode step.
* :func:`gdn_prefill` — chunked prefill over T tokens (tcgen05 tensor cores).
* :func:`kda_prefill` — KDA prefill over T tokens (state kept on chip).
* :func:`gdn_decode_ref` / :func:`kda_decode_ref` — the reference's 2-D
  (Q, K, V, Alpha|G, Beta, S_in, S_out, O) argument layout.
* :class:`ShardedGDNDecoder` — value-head-sharded decode over several GPUs
  with an optional NCCL all-gather of the outputs.

The importable module name is ``cuda_oxide_bench_b200`` (the directory name
has dashes; ``__graft_entry__.package()`` loads it).
"""
from ._lib import GDNError, LIB_PATH
from .api import (
    DecodeStep,
    check_device_status,
    gdn_decode,
    gdn_decode_ref,
    gdn_prefill,
    kda_decode,
    kda_prefill,
    kda_decode_ref,
    status_word,
)
from .sharded import ShardedGDNDecoder, shard_heads

__all__ = [
    "GDNError", "LIB_PATH", "DecodeStep", "check_device_status", "gdn_decode",
    "gdn_decode_ref", "gdn_prefill", "kda_decode", "kda_prefill", "kda_decode_ref", "status_word",
    "ShardedGDNDecoder", "shard_heads",
]
