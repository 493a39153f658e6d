"""Seeded synthetic workloads of the attention path, generated and encoded on the GPU through
the engine's own stores. Shared by ``bench.py`` and the full-size GPU tests.

The five named workloads restate the configurations the headline metric is quoted on:

* ``c1``  fp16 cache, 1 slot x 1 query token, 4096 rows
* ``c2``  fp8-e4m3 cache with per-(side, kv head) absmax scales, 1 slot x 6 draft lanes, 32768 rows
* ``c3``  turbo3 cache, 2 slots x 1 token, 131072 rows, 2 % of the channels scaled x8
* ``c4``  prefill: 8192 cached prefix rows + 16384 new tokens in 2048-token chunks, bf16-rounded
          values in an fp16 cache
* ``c5``  turbo3 cache, 8 slots x 6 lanes, 262144 rows per slot (split over the GPUs), outliers as c3

All shapes are GQA 24 query / 4 KV heads, head_dim 256, softmax scale 1/16.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import attn as A
from . import kv as K

N_Q, N_KV, HD, GQA = 24, 4, 256, 6
Q_STRIDE = 2 * HD            # interleaved [q | gate] per head
Q_ROW = N_Q * Q_STRIDE
OUT_ROW = N_Q * HD
SCALE = 1.0 / 16.0
ROW_BYTES = {K.KV_F16: 2048, K.KV_FP8: 1024, K.KV_T3: 400}
KIND_NAME = {K.KV_F16: "fp16", K.KV_FP8: "fp8-e4m3", K.KV_T3: "turbo3"}


@dataclass(frozen=True)
class Decode:
    """A decode / verify workload: `rows` is the context length per slot."""
    kvk: int
    slots: int
    lanes: int
    rows: int
    outlier_frac: float
    split_rows_over_ranks: bool = False     # strong scaling: the context is divided, not multiplied


DECODE = {
    "c1": Decode(K.KV_F16, 1, 1, 4096, 0.0),
    "c2": Decode(K.KV_FP8, 1, 6, 32768, 0.0),
    "c3": Decode(K.KV_T3, 2, 1, 131072, 0.02),
    "c5": Decode(K.KV_T3, 8, 6, 262144, 0.02, split_rows_over_ranks=True),
}
PREFILL_C4 = {"prefix": 8192, "new": 16384, "chunk": 2048}


@dataclass
class Cache:
    """One slot's paged K and V sides on the device."""
    kstore: torch.Tensor
    ktab: torch.Tensor
    vstore: torch.Tensor
    vtab: torch.Tensor
    rows: int
    kvk: int
    k_scale: torch.Tensor | None = None     # fp8: per-kv-head dequant scale (absmax / 448)
    v_scale: torch.Tensor | None = None

    def host_rows(self):
        """(k, v) as uint8 numpy [rows, row_bytes] in logical order (identity tables)."""
        rb = ROW_BYTES[self.kvk]
        return (self.kstore[: self.rows * rb].cpu().numpy().reshape(self.rows, rb),
                self.vstore[: self.rows * rb].cpu().numpy().reshape(self.rows, rb))


def outlier_multipliers(seed: int, frac: float, device) -> list[torch.Tensor]:
    """Per-(kv head, dim) channel multipliers for K and V: `frac` of the 1024 channels, chosen by
    `seed`, are scaled x8."""
    cg = torch.Generator(device="cpu")
    cg.manual_seed(seed + 7)
    out = []
    for _ in range(2):
        m = torch.ones(N_KV * HD, device=device)
        if frac > 0:
            n = max(1, int(round(frac * N_KV * HD)))
            m[torch.randperm(N_KV * HD, generator=cg)[:n].to(device)] = 8.0
        out.append(m)
    return out


def make_cache(kvk: int, rows: int, seed: int, outlier_frac: float, device,
               first_row: int = 0, same_v: bool = False) -> Cache:
    """Rows [first_row, first_row + rows) of a slot's cache (a rank's shard when first_row > 0 --
    the channel multipliers depend on the seed only, the row values on seed and first_row).
    Values are N(0,1), rounded through fp16, then stored as the kind demands."""
    rb = ROW_BYTES[kvk]
    npages = max((rows + 63) // 64, 1)
    kstore = torch.empty(npages * 64 * rb, dtype=torch.uint8, device=device)
    vstore = torch.empty(npages * 64 * rb, dtype=torch.uint8, device=device)
    ktab, vtab = K.mk_tab(kstore, rb, rows), K.mk_tab(vstore, rb, rows)
    g = torch.Generator(device=device)
    g.manual_seed(seed * 1000003 + first_row)
    mult = outlier_multipliers(seed, outlier_frac, device)
    v_row = torch.randn((1, N_KV * HD), generator=g, device=device).half().float()
    cache = Cache(kstore, ktab, vstore, vtab, rows, kvk)
    if kvk == K.KV_FP8:
        # per-(side, kv head) absmax over the whole cache: the whole slot is drawn at once
        assert rows <= 131072, "fp8 caches are generated in one piece"
        k = (torch.randn((rows, N_KV * HD), generator=g, device=device) * mult[0]).half().float()
        v = (torch.randn((rows, N_KV * HD), generator=g, device=device) * mult[1]).half().float()
        ka = k.view(rows, N_KV, HD).abs().amax(dim=(0, 2)).clamp_min(1e-30)
        va = v.view(rows, N_KV, HD).abs().amax(dim=(0, 2)).clamp_min(1e-30)
        ks, vs = ka / 448.0, va / 448.0
        A.kv_store_T((k.view(rows, N_KV, HD) / ks[None, :, None]).reshape(rows, -1).contiguous(),
                     (v.view(rows, N_KV, HD) / vs[None, :, None]).reshape(rows, -1).contiguous(),
                     ktab, vtab, 0, N_KV * HD, rows, fp8=True)
        cache.k_scale, cache.v_scale = ks, vs
    else:
        chunk = 8192
        for r0 in range(0, rows, chunk):
            t = min(chunk, rows - r0)
            k = (torch.randn((t, N_KV * HD), generator=g, device=device) * mult[0]).half().float()
            if same_v:
                v = v_row.expand(t, -1).contiguous()
            else:
                v = (torch.randn((t, N_KV * HD), generator=g, device=device) * mult[1]).half().float()
            if kvk == K.KV_T3:
                A.kv_store_T_t3(k, v, ktab, vtab, r0, N_KV, HD, t)
            else:
                A.kv_store_T(k, v, ktab, vtab, r0, N_KV * HD, t, fp8=False)
    torch.cuda.synchronize(device)
    return cache


def make_queries(nslots: int, lanes: int, seed: int) -> torch.Tensor:
    """Host fp32 [nslots, lanes, 24 * 512] N(0,1) (the gate half is drawn too and never read)."""
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    return torch.randn((nslots, lanes, N_Q * Q_STRIDE), generator=g)


def fold_k_scale(q: torch.Tensor, k_scale: torch.Tensor) -> torch.Tensor:
    """The reference's fp8 cache carries no scale (src/cuda_common.h:110-121): the K side's
    per-head scale is folded into Q by the caller. q [..., 24 * 512]."""
    qs = q.clone().view(*q.shape[:-1], N_Q, Q_STRIDE)
    qs[..., :HD] *= k_scale.to(q.device).repeat_interleave(GQA)[:, None]
    return qs.view(q.shape)


def apply_v_scale(out: torch.Tensor, v_scale: torch.Tensor) -> torch.Tensor:
    """... and the V side's into the output rows. out [..., 24 * 256]."""
    o = out.clone().view(*out.shape[:-1], N_Q, HD)
    o *= v_scale.to(out.device).repeat_interleave(GQA)[:, None]
    return o.view(out.shape)


def bf16_values(shape, generator, device) -> torch.Tensor:
    """N(0,1) rounded to bf16, magnitudes below 2^-14 flushed: exactly representable in fp16."""
    x = torch.randn(shape, generator=generator, device=device).bfloat16().float()
    return torch.where(x.abs() < 2.0 ** -14, torch.zeros_like(x), x)
