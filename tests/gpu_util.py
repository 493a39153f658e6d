"""Helpers that move a synthetic Case onto the GPU and drive the engine through the C ABI."""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

import q27_b200 as Q
from q27_b200 import _lib as L
from tests import synth
from tests.oracle_lib import REF_GPU_SO

SCALE = 1.0 / 16.0


class DeviceCase:
    def __init__(self, case: synth.Case, device, scatter_seed: int | None = None,
                 row_lo: int = 0, row_hi: int | None = None):
        """Upload rows [row_lo, row_hi) of the case's cache (a KV-sequence shard)."""
        self.case = case
        row_hi = case.rows if row_hi is None else row_hi
        self.row_lo, self.row_hi = row_lo, row_hi
        nrows = row_hi - row_lo
        perm = None
        if scatter_seed is not None:
            npages = max((nrows + 63) // 64, 1)
            perm = torch.from_numpy(np.random.default_rng(scatter_seed).permutation(npages))
        kb = torch.from_numpy(case.k[row_lo:row_hi].copy()).to(device)
        vb = torch.from_numpy(case.v[row_lo:row_hi].copy()).to(device)
        if nrows == 0:
            kb = torch.zeros((0, case.k.shape[1]), dtype=torch.uint8, device=device)
            vb = torch.zeros((0, case.v.shape[1]), dtype=torch.uint8, device=device)
        self.kside = Q.paged_from_rows(kb, case.kvk, page_perm=perm)
        self.vside = Q.paged_from_rows(vb, case.kvk, page_perm=perm, is_v=True)
        ntok = len(case.pos)
        self.ntok = ntok
        self.q = [torch.from_numpy(case.q[t].copy()).to(device) for t in range(ntok)]
        self.pos = [torch.tensor([p], dtype=torch.int32, device=device) for p in case.pos]
        self.out = [torch.full((synth.OUT_ROW,), float("nan"), device=device) for _ in range(ntok)]
        # NaN-poisoned scratch: nothing may depend on its initial contents
        self.scratch = torch.full((Q.decode_scratch_floats(ntok),), float("nan"), device=device)

    def slot(self) -> Q.SlotArgs:
        return Q.SlotArgs(self.kside.tab, self.vside.tab, self.q, self.pos, self.out, self.scratch,
                          row_base=self.row_lo,
                          row_count=(self.row_hi - self.row_lo) if (self.row_lo or self.row_hi != self.case.rows) else 2**31 - 1)

    def run3(self, exact=False):
        if exact:
            Q.attn_decode_batched([self.slot()], synth.Q_STRIDE, 24, 4, 256, SCALE,
                                  kvk=self.case.kvk, exact=True)
        else:
            Q.attn_decode3(self.q, synth.Q_STRIDE, self.kside.tab, self.vside.tab, self.out,
                           self.scratch, self.pos, 0, 24, 4, 256, SCALE, ntok=self.ntok,
                           kvk=self.case.kvk)
        torch.cuda.synchronize()
        return np.stack([o.cpu().numpy() for o in self.out])


class RefGpu:
    """The reference's own kernels recompiled for sm_100a (oracle/_ref), if present."""

    def __init__(self):
        if not REF_GPU_SO.exists():
            raise FileNotFoundError(REF_GPU_SO)
        self.lib = C.CDLL(str(REF_GPU_SO))
        vp, i, f = C.c_void_p, C.c_int, C.c_float
        self.lib.q27ref_attn_decode3.argtypes = [vp, i, vp, vp, vp, vp, vp, i, i, i, f, vp, i, i, i]
        self.lib.q27ref_attn_decode3.restype = None
        self.lib.q27ref_attn_prefill_T.argtypes = [vp, i, i, vp, vp, vp, i, vp, i, i, i, i, i, i, f,
                                                   vp, i]
        self.lib.q27ref_attn_prefill_T.restype = None
        self.lib.q27ref_kv_store_T_t3.argtypes = [vp, vp, vp, vp, i, i, i, i, vp, i]
        self.lib.q27ref_kv_store_T_t3.restype = None
        self.lib.q27ref_wht_T.argtypes = [vp, i, i, i, i, i, i, vp]
        self.lib.q27ref_wht_T.restype = None

    def decode3(self, dc: DeviceCase, fd2_only=True):
        n = dc.ntok
        qa = (C.c_void_p * 16)(*[t.data_ptr() for t in dc.q])
        oa = (C.c_void_p * 16)(*[t.data_ptr() for t in dc.out])
        pa = (C.c_void_p * 16)(*[t.data_ptr() for t in dc.pos])
        self.lib.q27ref_attn_decode3(qa, synth.Q_STRIDE, dc.kside.tab.data_ptr(),
                                     dc.vside.tab.data_ptr(), oa, dc.scratch.data_ptr(), pa, 24, 4,
                                     256, SCALE, None, n, dc.case.kvk, int(fd2_only))
        torch.cuda.synchronize()
        return np.stack([o.cpu().numpy() for o in dc.out])
