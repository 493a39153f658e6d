"""The decode entry point that takes no scratch buffer, for callers that cannot provide one
(no allocator of their own, or running where device allocation is not allowed). Its split
partials live in an array inside the library instead of caller memory. Collected last on
purpose: a run that stops at the first failure has then already run every other test.

The check: through the C ABI, two calls in a row must each reproduce what the ordinary
entry point (caller-provided scratch) writes for the same inputs, within the suite's
parity tolerance, and sizes past the built-in capacity must be refused cleanly."""
import ctypes as C

import numpy as np
import pytest
import torch

import q27_b200 as Q
from q27_b200 import _lib as L
from tests import synth
from tests.gpu_util import SCALE, DeviceCase
from tests.oracle_lib import KV_F16, KV_T3

pytestmark = pytest.mark.gpu


def p3(tensors):
    p = L.P3()
    for i, t in enumerate(tensors):
        p.p[i] = t.data_ptr()
    return p


@pytest.mark.parametrize("kvk,rows,pos", [(KV_T3, 3000, [2999, 2998, 1500]), (KV_F16, 900, [899])])
def test_no_alloc_entry_matches_regular_entry_twice(oracle, cuda, kvk, rows, pos):
    c = synth.make_case(oracle, kvk, rows=rows, pos=pos, seed=91, outlier_frac=0.02 if kvk == KV_T3 else 0.0)
    dc = DeviceCase(c, cuda)
    want = dc.run3()                                   # ordinary entry, caller's scratch
    oracle_out = oracle.attn_decode(c.q, c.k, c.v, kvk, c.pos)
    assert synth.tolerance_ok(want, oracle_out)[0]
    lib = L.lib()
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):                              # the array keeps the last call's contents
        for o in dc.out:
            o.fill_(float("nan"))
        q, o, p = p3(dc.q), p3(dc.out), p3(dc.pos)
        rc = lib.q27_attn_decode3_noalloc(C.byref(q), synth.Q_STRIDE, dc.kside.tab.data_ptr(),
                                          dc.vside.tab.data_ptr(), C.byref(o), C.byref(p), 24, 4,
                                          256, SCALE, stream, len(pos), kvk)
        assert rc == L.OK, lib.q27_status_string(rc)
        torch.cuda.synchronize()
        got = np.stack([t.cpu().numpy() for t in dc.out])
        ok, excess, rel = synth.tolerance_ok(got, want)
        assert ok, (call, excess, rel)
        # a second, shorter problem in between must not leave anything behind that matters
        for t, newp in enumerate(pos):
            dc.pos[t].fill_(max(newp // 3, 0) if call == 0 else newp)
        if call == 0:
            rc = lib.q27_attn_decode3_noalloc(C.byref(q), synth.Q_STRIDE, dc.kside.tab.data_ptr(),
                                              dc.vside.tab.data_ptr(), C.byref(o), C.byref(p), 24,
                                              4, 256, SCALE, stream, len(pos), kvk)
            assert rc == L.OK
            torch.cuda.synchronize()
            for t, newp in enumerate(pos):
                dc.pos[t].fill_(newp)


def test_no_alloc_entry_refuses_sizes_past_its_capacity(oracle, cuda):
    c = synth.make_case(oracle, KV_F16, rows=64, pos=[63] * 5, seed=92)
    dc = DeviceCase(c, cuda)
    q, o, p = p3(dc.q), p3(dc.out), p3(dc.pos)
    rc = L.lib().q27_attn_decode3_noalloc(C.byref(q), synth.Q_STRIDE, dc.kside.tab.data_ptr(),
                                          dc.vside.tab.data_ptr(), C.byref(o), C.byref(p), 24, 4,
                                          256, SCALE, None, L.NOALLOC_MAX_LANES + 1, KV_F16)
    assert rc == L.ERR_TOO_LARGE
    torch.cuda.synchronize()
    assert all(torch.isnan(t).all() for t in dc.out)   # refused means nothing ran
