"""CPU restatement (numpy) of the KV section of the reference's prefix snapshots and of the
identity of a snapshot entry. TEST INFRASTRUCTURE ONLY: imported by tests/ alone; nothing under
q27_b200/ loads it.

Follows src/prefix_cache.h:44-82 (pfx_fnv1a64, pfx_compat_hash, PfxHdr, PFX_MAGIC / PFX_VERSION),
:224-248 (the entry file: header, tokens, state) and src/engine.cuh:3727-3731, 3786-3822
(pfx_kv_bytes; pfx_export's walk: per pair the K rows [0, n) then the V rows [0, n) in logical
order, the last pair one row longer). Pinned against the reference's own header compiled from
the reference tree (oracle/_ref, tests/test_snapshot_cpu.py) and the fixture
tests/golden/pfx_identity.npz generated from it."""
from __future__ import annotations

import struct

import numpy as np

FNV_SEED = 1469598103934665603        # src/prefix_cache.h:44 (the reference's own basis)
FNV_PRIME = 1099511628211
MASK = (1 << 64) - 1
PFX_MAGIC, PFX_VERSION = 0x50373251, 1


def fnv1a64(data: bytes, h: int = FNV_SEED) -> int:
    for b in data:                      # src/prefix_cache.h:46-49
        h = ((h ^ b) * FNV_PRIME) & MASK
    return h


def compat_hash(model_path: str, model_bytes: int, n_layer: int, n_kv: int, head_dim: int,
                gdn_heads: int, gdn_dim: int, gdn_ch: int, kv_kind: int, format_version: int) -> int:
    h = fnv1a64(model_path.encode())    # src/prefix_cache.h:56-62: then nine int64 values
    v = struct.pack("<9q", model_bytes, n_layer, n_kv, head_dim, gdn_heads, gdn_dim, gdn_ch,
                    kv_kind, format_version)
    return fnv1a64(v, h)


def header(compat: int, tokens, L: int, gdn_bytes: int, kv_bytes: int) -> bytes:
    """PfxHdr as PrefixCache::write fills it (src/prefix_cache.h:66-80, 241-248): packed,
    little-endian, 64 bytes."""
    key = fnv1a64(np.asarray(tokens[:L], dtype="<i4").tobytes())
    return struct.pack("<IIQQiiQQQQ", PFX_MAGIC, PFX_VERSION, compat, key, L, 0, gdn_bytes, kv_bytes, 0, 0)


def kv_bytes(L: int, n_attn_pairs: int, k_row: int, v_row: int) -> int:
    """pfx_kv_bytes (src/engine.cuh:3727-3731)."""
    return L * n_attn_pairs * (k_row + v_row) + (L + 1) * (k_row + v_row)


def kv_blob(k_rows: list, v_rows: list, L: int, extra: list) -> np.ndarray:
    """k_rows[c] / v_rows[c]: uint8 [rows, row_bytes] logical rows of pair c. The blob of
    pfx_export: pair by pair, K rows [0, L + extra[c]) then V rows [0, L + extra[c])."""
    out = []
    for c in range(len(k_rows)):
        n = L + extra[c]
        out.append(np.ascontiguousarray(k_rows[c][:n]).reshape(-1))
        out.append(np.ascontiguousarray(v_rows[c][:n]).reshape(-1))
    return np.concatenate(out) if out else np.zeros(0, np.uint8)
