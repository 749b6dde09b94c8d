"""ffa_align_noalloc: alignment for callers that cannot allocate device memory.

Callers running inside a framework that owns every device allocation, or in a
pipeline whose memory is fixed at start-up, cannot let the aligner call
cudaMalloc.  ffa_align_noalloc runs the same path as ffa_align with its
scratch in buffers built into the library.  These tests call it through the
C ABI and check that it returns exactly what ffa_align returns, on two calls
in a row (the second reuses the first call's scratch), that a repeated call
takes no device memory, and that a batch too large for the built-in scratch
is refused with a clear error.  This file is collected last on purpose.
"""
import ctypes

import numpy as np
import pytest
import torch

import fast_forced_aligner_b200 as ffa
from fast_forced_aligner_b200 import workloads
from fast_forced_aligner_b200.build import LIB
from tests.helpers import assert_same_bits, cuda_records

pytestmark = pytest.mark.gpu


class Record(ctypes.Structure):
    _fields_ = [("emissions", ctypes.c_void_p), ("targets", ctypes.c_void_p),
                ("frames", ctypes.c_int64), ("vocab", ctypes.c_int32), ("tokens", ctypes.c_int32),
                ("blank", ctypes.c_int32), ("reserved", ctypes.c_int32)]


class Outputs(ctypes.Structure):
    _fields_ = [(name, ctypes.c_void_p) for name in (
        "labels", "scores", "status", "objective", "stitched", "repair_passes", "repaired_frames",
        "shortcut_stats", "routing_stats", "reuse_stats")]


def library():
    lib = ctypes.CDLL(str(LIB))
    lib.ffa_last_error.restype = ctypes.c_char_p
    lib.ffa_align_noalloc.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_int,
                                      ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    lib.ffa_align_noalloc.restype = ctypes.c_int
    return lib


def records_of(es, ts, blank):
    return (Record * len(es))(*[Record(e.data_ptr(), t.data_ptr() if t.numel() else None, e.shape[0],
                                       e.shape[1], t.numel(), blank, 0) for e, t in zip(es, ts)])


def noalloc(lib, es, ts, blank, mode):
    """One ffa_align_noalloc call with caller-allocated outputs."""
    B, N = len(es), sum(e.shape[0] for e in es)
    dev = es[0].device
    out = {"labels": torch.empty(N, dtype=torch.int64, device=dev),
           "scores": torch.empty(N, dtype=torch.float32, device=dev),
           "status": torch.empty(B, dtype=torch.int32, device=dev),
           "objective": torch.empty(B, dtype=torch.float32, device=dev),
           "stitched": torch.empty(B, dtype=torch.int32, device=dev),
           "repair_passes": torch.empty(B, dtype=torch.int32, device=dev),
           "repaired_frames": torch.empty(B, dtype=torch.int64, device=dev),
           "shortcut_stats": torch.empty(B, 3, dtype=torch.int64, device=dev),
           "routing_stats": torch.empty(B, 3, dtype=torch.int32, device=dev)}
    outs = Outputs(*[out[k].data_ptr() for k in out], None)
    recs = records_of(es, ts, blank)
    rc = lib.ffa_align_noalloc(ctypes.cast(recs, ctypes.c_void_p), B, 0 if mode == "conventional" else 1,
                               1, None, ctypes.addressof(outs),
                               ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, lib.ffa_last_error()
    return out, recs


def check_same(out, expected, what):
    for name in ("labels", "scores", "status", "objective"):
        assert_same_bits(out[name].cpu().numpy(), getattr(expected, name).cpu().numpy(), f"{what} {name}")


@pytest.mark.parametrize("mode", ["conventional", "optimized"])
def test_noalloc_matches_align_on_two_calls_in_a_row(cuda, mode):
    lib = library()
    first = workloads.config(0)
    second = workloads.config(1, scale=0.25)
    e1, t1 = cuda_records(*first.records())
    e2, t2 = cuda_records(*second.records())
    want1 = ffa.align(e1, t1, blank_id=first.blank, mode=mode)
    want2 = ffa.align(e2, t2, blank_id=second.blank, mode=mode)
    got1, _ = noalloc(lib, e1, t1, first.blank, mode)
    got2, _ = noalloc(lib, e2, t2, second.blank, mode)
    torch.cuda.synchronize()
    check_same(got1, want1, "first call")
    check_same(got2, want2, "second call")
    assert (got1["status"] == 0).all() and (got2["status"] == 0).all()


def test_repeated_noalloc_call_takes_no_device_memory(cuda):
    lib = library()
    wl = workloads.config(0)
    es, ts = cuda_records(*wl.records())
    noalloc(lib, es, ts, wl.blank, "conventional")  # first call on the device: set-up
    torch.cuda.synchronize()
    B, N = len(es), sum(e.shape[0] for e in es)
    outs_t = [torch.empty(N, dtype=torch.int64, device=cuda), torch.empty(N, dtype=torch.float32, device=cuda)] + \
             [torch.empty(B, dtype=torch.int32, device=cuda) for _ in range(4)] + \
             [torch.empty(B, dtype=torch.int64, device=cuda), torch.empty(B, 3, dtype=torch.int64, device=cuda),
              torch.empty(B, 3, dtype=torch.int32, device=cuda)]
    outs = Outputs(outs_t[0].data_ptr(), outs_t[1].data_ptr(), outs_t[2].data_ptr(), outs_t[3].data_ptr(),
                   outs_t[4].data_ptr(), outs_t[5].data_ptr(), outs_t[6].data_ptr(), outs_t[7].data_ptr(),
                   outs_t[8].data_ptr(), None)
    recs = records_of(es, ts, wl.blank)
    torch.cuda.synchronize()
    free_before, _ = torch.cuda.mem_get_info()
    rc = lib.ffa_align_noalloc(ctypes.cast(recs, ctypes.c_void_p), B, 0, 1, None, ctypes.addressof(outs),
                               ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    free_after, _ = torch.cuda.mem_get_info()
    assert rc == 0, lib.ffa_last_error()
    assert free_after == free_before
    assert (outs_t[2] == 0).all()


def test_batch_beyond_the_builtin_scratch_is_refused(cuda):
    lib = library()
    # Planning never dereferences device pointers: aligned fake addresses do.
    B = 512
    recs = (Record * B)(*[Record(0x100000 * (i + 1), 0x90000000 + 0x10000 * i, 4000, 32, 1500, 0, 0)
                          for i in range(B)])
    outs = Outputs(*([0x1000] * 9), None)
    rc = lib.ffa_align_noalloc(ctypes.cast(recs, ctypes.c_void_p), B, 0, 1, None, ctypes.addressof(outs),
                               None)
    assert rc == -2  # FFA_ERR_UNSUPPORTED
    assert b"scratch" in lib.ffa_last_error()
