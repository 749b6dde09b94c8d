"""The native boundary without a GPU: library loading, exported symbols,
host-side planning and the Python surface's argument contract."""
import ctypes
import re
from pathlib import Path

import numpy as np
import pytest
import torch
from torch.utils import cpp_extension

import fast_forced_aligner_b200 as ffa
from fast_forced_aligner_b200 import alignment

ROOT = Path(__file__).resolve().parents[1]
LIB = ROOT / "fast_forced_aligner_b200" / "libffa_b200.so"
SHIM = ROOT / "fast_forced_aligner_b200" / "_ffa_torch.so"


class Record(ctypes.Structure):
    _fields_ = [("emissions", ctypes.c_void_p), ("targets", ctypes.c_void_p),
                ("frames", ctypes.c_int64), ("vocab", ctypes.c_int32), ("tokens", ctypes.c_int32),
                ("blank", ctypes.c_int32), ("format", ctypes.c_int32)]


class Sizes(ctypes.Structure):
    _fields_ = [("staging_bytes", ctypes.c_size_t), ("workspace_bytes", ctypes.c_size_t),
                ("total_frames", ctypes.c_int64)]


@pytest.fixture(scope="module")
def lib():
    if not LIB.exists():
        from fast_forced_aligner_b200 import build
        build.build()
    handle = ctypes.CDLL(str(LIB))
    handle.ffa_last_error.restype = ctypes.c_char_p
    return handle


def declared_symbols():
    names = []
    for header in (ROOT / "include").glob("*.h"):
        names += re.findall(r"FFA_API\s+[\w\s\*]+?\b(ffa_\w+)\s*\(", header.read_text())
    return sorted(set(names))


def test_library_exports_every_declared_symbol(lib):
    names = declared_symbols()
    assert {"ffa_align", "ffa_align_query", "ffa_emission_validity"} <= set(names)
    for name in names:
        assert hasattr(lib, name), name
    assert lib.ffa_abi_version() == 2


def records(*specs, fmt=0):
    arr = (Record * len(specs))()
    for i, (T, V, U, blank) in enumerate(specs):
        # Planning never dereferences device pointers: fake aligned addresses.
        arr[i] = Record(0x10000 * (i + 1), 0x900000 * (i + 1) if U else None, T, V, U, blank, fmt)
    return arr


def test_align_query_sizes(lib):
    recs = records((600, 32, 100, 0), (7, 6, 0, 5), (2305, 1025, 2047, 1024))
    sizes = Sizes()
    assert lib.ffa_align_query(recs, 3, 0, 1, ctypes.byref(sizes)) == 0
    assert sizes.total_frames == 600 + 7 + 2305
    assert sizes.staging_bytes > 0 and sizes.staging_bytes % 256 == 0
    # Workspace holds at least 2 bits per DP cell (T*S/4 bytes).
    assert sizes.workspace_bytes >= (600 * 201 + 7 + 2305 * 4095) // 4


def test_align_query_sizes_long_records(lib):
    # 32767 tokens (65535 states, a 16-CTA cluster): backpointers alone take
    # 2 bits per cell.
    recs = records((34000, 32, 32767, 0), (90000, 32, 27000, 0))
    sizes = Sizes()
    assert lib.ffa_align_query(recs, 2, 1, 1, ctypes.byref(sizes)) == 0
    assert sizes.total_frames == 34000 + 90000
    assert sizes.workspace_bytes >= (34000 * 65535 + 90000 * 54001) // 4


def test_window_codes_arena_only_for_throughput_bound_batches(lib):
    # Optimized mode gives records of at most 2048 frames to the window route
    # when there are more than 4 per SM.  Up to 8 per SM their codes stay in
    # shared memory; beyond that the workspace carries a global codes arena
    # of 32 B per frame plus 256 B per record.  (Planning without a GPU
    # assumes a B200's 148 SMs.)
    def extra(n):
        recs = records(*[(600, 32, 100, 0)] * n)
        opt, conv = Sizes(), Sizes()
        assert lib.ffa_align_query(recs, n, 1, 1, ctypes.byref(opt)) == 0
        assert lib.ffa_align_query(recs, n, 0, 1, ctypes.byref(conv)) == 0
        return opt.workspace_bytes - conv.workspace_bytes, 600 * n
    latency_bound, frames = extra(600)      # 5 window records per SM
    assert latency_bound < 32 * frames
    throughput_bound, frames = extra(1200)  # 9 per SM
    assert throughput_bound >= 32 * frames + 256 * 1200


@pytest.mark.parametrize("spec, code", [
    ((0, 32, 1, 0), -2), ((10, 0, 1, 0), -2), ((10, 8193, 1, 0), -2),
    ((10, 32, 32768, 0), -2), ((10, 32, 1, 32), -2), ((10, 32, 1, -1), -2),
])
def test_align_query_rejects_unsupported_metadata(lib, spec, code):
    sizes = Sizes()
    assert lib.ffa_align_query(records(spec), 1, 0, 1, ctypes.byref(sizes)) == code
    assert lib.ffa_last_error()


def test_align_query_rejects_malformed_calls(lib):
    sizes = Sizes()
    assert lib.ffa_align_query(records((10, 32, 1, 0)), 0, 0, 1, ctypes.byref(sizes)) == -1
    assert lib.ffa_align_query(records((10, 32, 1, 0)), 1, 7, 1, ctypes.byref(sizes)) == -1
    assert lib.ffa_align_query(records((10, 32, 1, 0)), 1, 0, 8, ctypes.byref(sizes)) == -1
    missing = records((10, 32, 3, 0))
    missing[0].targets = None
    assert lib.ffa_align_query(missing, 1, 0, 1, ctypes.byref(sizes)) == -1
    unaligned = records((10, 32, 1, 0))
    unaligned[0].emissions = 0x10002
    assert lib.ffa_align_query(unaligned, 1, 0, 1, ctypes.byref(sizes)) == -1


def test_align_reports_small_buffers_before_any_device_work(lib):
    recs = records((100, 32, 10, 0))
    sizes = Sizes()
    assert lib.ffa_align_query(recs, 1, 0, 1, ctypes.byref(sizes)) == 0
    outs = (ctypes.c_void_p * 10)(*([0x1000] * 10))
    staging = ctypes.create_string_buffer(8)
    rc = lib.ffa_align(recs, ctypes.c_int64(1), 0, 1, None, outs, staging, ctypes.c_size_t(8),
                       ctypes.c_void_p(0x100000), ctypes.c_size_t(sizes.workspace_bytes), None)
    assert rc == -3
    assert b"staging" in lib.ffa_last_error()


def test_validity_and_target_queries(lib):
    sizes = Sizes()
    assert lib.ffa_emission_validity_query(records((100, 32, 0, 0), (5, 3, 0, 0)), 2,
                                           ctypes.byref(sizes)) == 0
    assert sizes.total_frames == 105 and sizes.workspace_bytes >= sizes.staging_bytes
    assert lib.ffa_check_targets_query(records((100, 32, 5, 0)), 1, ctypes.byref(sizes)) == 0


def test_logits_formats_plan_like_log_probabilities(lib):
    # Formats 1 (fp32 logits) and 2 (bf16 logits) plan the same DP; the
    # workspace also holds one fp32 log-sum-exp per frame.
    specs = ((600, 32, 100, 0), (7, 6, 0, 5), (2305, 1025, 2047, 1024))
    base, f32, bf16 = Sizes(), Sizes(), Sizes()
    assert lib.ffa_align_query(records(*specs), 3, 1, 1, ctypes.byref(base)) == 0
    assert lib.ffa_align_query(records(*specs, fmt=1), 3, 1, 1, ctypes.byref(f32)) == 0
    assert lib.ffa_align_query(records(*specs, fmt=2), 3, 1, 1, ctypes.byref(bf16)) == 0
    assert f32.total_frames == bf16.total_frames == base.total_frames
    assert f32.workspace_bytes == bf16.workspace_bytes >= base.workspace_bytes + 4 * base.total_frames
    assert f32.staging_bytes == base.staging_bytes


def test_input_format_rules(lib):
    sizes = Sizes()
    # A bf16 record needs 2-byte alignment only; fp32 ones need 4.
    half = records((10, 33, 1, 0), fmt=2)
    half[0].emissions = 0x10002
    assert lib.ffa_align_query(half, 1, 1, 1, ctypes.byref(sizes)) == 0
    single = records((10, 33, 1, 0), fmt=1)
    single[0].emissions = 0x10002
    assert lib.ffa_align_query(single, 1, 1, 1, ctypes.byref(sizes)) == -1
    odd = records((10, 33, 1, 0), fmt=2)
    odd[0].emissions = 0x10001
    assert lib.ffa_align_query(odd, 1, 1, 1, ctypes.byref(sizes)) == -1
    # Unknown formats, and formats mixed in one call, are rejected.
    assert lib.ffa_align_query(records((10, 32, 1, 0), fmt=3), 1, 1, 1, ctypes.byref(sizes)) == -1
    assert b"format" in lib.ffa_last_error()
    mixed = records((10, 32, 1, 0), (12, 32, 1, 0), fmt=1)
    mixed[1].format = 2
    assert lib.ffa_align_query(mixed, 2, 1, 1, ctypes.byref(sizes)) == -1
    assert b"same input format" in lib.ffa_last_error()
    # The emission-validity scan reads fp32 only.
    assert lib.ffa_emission_validity_query(records((10, 32, 0, 0), fmt=1), 1, ctypes.byref(sizes)) == 0
    assert lib.ffa_emission_validity_query(records((10, 32, 0, 0), fmt=2), 1, ctypes.byref(sizes)) == -2


def test_row_logsumexp_query(lib):
    sizes = Sizes()
    assert lib.ffa_row_logsumexp_query(records((100, 32, 0, 0), (5, 1025, 0, 0), fmt=2), 2,
                                       ctypes.byref(sizes)) == 0
    assert sizes.total_frames == 105 and sizes.workspace_bytes >= sizes.staging_bytes > 0
    assert lib.ffa_row_logsumexp_query(records((100, 32, 0, 0)), 1, ctypes.byref(sizes)) == -1
    assert b"logits" in lib.ffa_last_error()


def test_torch_ops_register_without_a_gpu():
    torch.ops.load_library(str(SHIM))
    for name in ("align", "align_packed", "emission_validity", "check_targets", "token_spans",
                 "row_logsumexp", "align_stream"):
        assert hasattr(torch.ops.ffa_b200, name)
    schema = str(torch.ops.ffa_b200.align.default._schema)
    assert "int fmt=0" in schema


# ---- Python surface (reference tests/test_extension.py, test_core.py:85-93) ----

@pytest.fixture()
def fresh_loader():
    alignment.load_extension.cache_clear()
    yield
    alignment.load_extension.cache_clear()


def test_cpu_torch_reports_cuda_requirement(monkeypatch, fresh_loader):
    monkeypatch.setattr(torch.version, "cuda", None)
    with pytest.raises(RuntimeError, match="CUDA-enabled PyTorch"):
        ffa.load_extension()


def test_missing_gpu_reports_driver_requirement(monkeypatch, fresh_loader):
    monkeypatch.setattr(torch.version, "cuda", "12.8")
    monkeypatch.setattr(torch.cuda, "is_available", lambda: False)
    with pytest.raises(RuntimeError, match="accessible NVIDIA GPU"):
        ffa.load_extension()


@pytest.mark.parametrize("toolkit", [None, "/nonexistent/cuda-toolkit"])
def test_unbuilt_library_without_toolkit_reports_nvcc(monkeypatch, fresh_loader, toolkit, tmp_path):
    monkeypatch.setattr(torch.version, "cuda", "12.8")
    monkeypatch.setattr(torch.cuda, "is_available", lambda: True)
    monkeypatch.setattr(cpp_extension, "CUDA_HOME", toolkit)
    monkeypatch.setattr(alignment, "_PACKAGE", tmp_path)  # no built library there
    with pytest.raises(RuntimeError, match="including nvcc"):
        ffa.load_extension()


def test_argument_contract_without_gpu():
    e = torch.zeros(12, 6)
    t = torch.tensor([1])
    with pytest.raises(ValueError, match="mode"):
        ffa.align([e], [t], mode="unknown")
    with pytest.raises(TypeError, match="check_inputs"):
        ffa.align([e], [t], check_inputs=1)
    with pytest.raises(ValueError):
        ffa.align([], [])
    with pytest.raises(ValueError):
        ffa.align([e], [])
    with pytest.raises(ValueError, match="blank"):
        ffa.align([e], [t], blank_id=[0, 1])
    with pytest.raises(TypeError):  # the reference's list(True) raises TypeError too
        ffa.align([e], [t], blank_id=True)
    with pytest.raises(ValueError):
        ffa.align([e], [t], blank_id=[True])
    with pytest.raises(ValueError, match="CUDA"):
        ffa.align([e], [t])  # CPU tensors
    with pytest.raises(TypeError, match="from_logits"):
        ffa.align([e], [t], from_logits=1)
    with pytest.raises(TypeError, match="from_logits"):
        ffa.align_packed(e, [12], t, [1], from_logits="yes")
    with pytest.raises(ValueError, match="CUDA"):
        ffa.row_logsumexp(e)
    with pytest.raises(ValueError):
        ffa.emission_validity([])
    with pytest.raises(ValueError):
        ffa.emission_validity([e])


def test_packed_argument_contract_without_gpu():
    e = torch.zeros(12, 6)
    t = torch.tensor([1, 2])
    with pytest.raises(ValueError, match="frames"):
        ffa.align_packed(e, [6.0, 6.0], t, [1, 1])
    with pytest.raises(ValueError, match="tokens"):
        ffa.align_packed(e, [6, 6], t, np.array([[1, 1]]))
    with pytest.raises(ValueError, match="matching"):
        ffa.align_packed(e, [6, 6], t, [2])
    with pytest.raises(ValueError, match="matching"):
        ffa.align_packed(e, [], t, [])
    with pytest.raises(ValueError, match="blank"):
        ffa.align_packed(e, [6, 6], t, [1, 1], blank_id=[0])
    with pytest.raises(TypeError):
        ffa.align_packed(e, [6, 6], t, [1, 1], blank_id=True)
    with pytest.raises(ValueError, match="frames"):
        ffa.align_packed(e, torch.tensor([6.0, 6.0]), t, [1, 1])
    with pytest.raises(ValueError, match="mode"):
        ffa.align_packed(e, [6, 6], t, [1, 1], mode="fast")
    with pytest.raises(ValueError, match="CUDA"):
        ffa.align_packed(e, np.array([6, 6]), t, torch.tensor([1, 1]), blank_id=np.array([0, 0]))
