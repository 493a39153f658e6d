"""q27_b200 -- a B200 (sm_100a) attention engine behind the kernel-launch surface of
signalnine/q27's full-attention layers: split-KV flash-decode, shared-KV MTP verify,
causal GQA prefill over a reused prefix, all over fp16 / fp8-e4m3 / turbo3 paged KV (plus the
turbo3v / turbo5k / int8-g64 kinds, whose K side differs, through the fp32 kernels).

The compute path is hand-written CUDA reached through a C ABI (include/q27_b200.h);
this package is the thin host-side mirror of the reference's launch functions."""
from . import _lib
from .kv import (KV_F16, KV_FP8, KV_T3, KV_T3V, KV_T5K, KV_I8G64, KV_PAGE, KIND_NAMES, KvPool, PagedSide, kv_k_rotated, mk_tab,
                 paged_from_rows, row_bytes)
from .attn import (BatchedDecode, SlotArgs, marshal_slots, attn_decode, attn_decode3, attn_decode3_noalloc, attn_decode_batched,
                   attn_decode_partial, attn_decode_partial_push, attn_decode_exchange, attn_merge_partials,
                   attn_merge_pushed, attn_prefill_T, attn_verify_partials, launch_count,
                   decode_scratch_floats, kv_dequant, kv_store3, kv_store_T, kv_store_T_t3,
                   kv_store_t3, kv_store_lanes_shard, kv_store_rows_shard, wht3,
                   prefill_part_floats, wht_T)
from .snapshot import KvLineage

__all__ = [n for n in dir() if not n.startswith("_")]
