"""CPU tests of the drop-in boundary: the C ABI library loads and exports every
symbol include/fa_sm100.h declares, argument validation that needs no GPU,
and the torch extension's names and error messages (reference
csrc/bindings.cpp:70-141, csrc/tensorcore_attention.cu:2731-2823)."""

import ctypes
import re
from pathlib import Path

import pytest
import torch

from flash_attention_2_lab_b200 import _native

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "fa_sm100.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(fa_\w+)\s*\(", text)))


def test_header_declares_expected_entry_points():
    names = declared_functions()
    for n in ("fa_fwd_sm100", "fa_fwd_sm100_varlen", "fa_last_error", "fa_read_status"):
        assert n in names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(_native.LIB_PATH))
    for name in declared_functions():
        assert hasattr(lib, name), f"{name} declared in fa_sm100.h but not exported"
    assert set(declared_functions()) == set(_native.ABI)


def test_invalid_sizes_rejected_without_gpu():
    lib = _native.lib()
    rc = lib.fa_fwd_sm100(None, None, None, None, -1, 1, 128, 0, 0.125, None)
    assert rc == -1
    assert "negative" in _native.last_error()
    rc = lib.fa_fwd_sm100_varlen(None, None, None, None, 1, 1, -5, 4, 0, 0.125, None)
    assert rc == -1


def test_empty_problem_is_noop_without_gpu():
    lib = _native.lib()
    assert lib.fa_fwd_sm100(None, None, None, None, 0, 8, 128, 1, 0.125, None) == 0
    assert lib.fa_fwd_sm100(None, None, None, None, 2, 8, 0, 0, 0.125, None) == 0


def test_null_and_misaligned_pointers_rejected():
    lib = _native.lib()
    assert lib.fa_fwd_sm100(None, None, None, None, 1, 1, 128, 0, 0.125, None) == -1
    assert "null" in _native.last_error()
    rc = lib.fa_fwd_sm100(8, 16, 32, 48, 1, 1, 128, 0, 0.125, None)
    assert rc == -1 and "aligned" in _native.last_error()


def test_bad_scale_rejected():
    lib = _native.lib()
    rc = lib.fa_fwd_sm100(16, 16, 16, 16, 1, 1, 128, 0, float("nan"), None)
    assert rc == -1 and "scale" in _native.last_error()


def test_smem_footprint_fits_b200():
    assert 0 < _native.lib().fa_smem_bytes() <= 227 * 1024


REFERENCE_NAMES = [
    "tensorcore_attention_forward_production_128x128",
    "tensorcore_attention_forward",
    "tensorcore_attention_forward_bc32",
    "tensorcore_attention_forward_bc32_raw_pv",
    "tensorcore_attention_forward_bc32_raw_qk_raw_pv",
]


def test_extension_exposes_reference_entry_points():
    ext = _native.ext()
    for n in REFERENCE_NAMES + ["attention_forward"]:
        assert callable(getattr(ext, n))


def test_extension_rejects_cpu_tensors_with_reference_message():
    ext = _native.ext()
    x = torch.zeros(1, 1, 128, 64, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="query must be a CUDA tensor"):
        ext.tensorcore_attention_forward_production_128x128(x, x, x, False)
    with pytest.raises(RuntimeError, match="query must be a CUDA tensor"):
        ext.attention_forward(x, x, x, True, None)


def test_package_api_names():
    import flash_attention_2_lab_b200 as fa

    for n in ("attention_forward", "attention_forward_causal",
              "tensorcore_attention_forward_production_128x128"):
        assert callable(getattr(fa, n))


def test_drop_in_module_shim():
    import flash_attention_cuda

    assert callable(flash_attention_cuda.tensorcore_attention_forward_production_128x128)


def test_policy_setters_race_free_with_validating_calls():
    # One thread flips the process-wide policies (atomic settings) while
    # another runs the ABI's argument validation; neither may crash, and
    # every validating call keeps its own error code and per-thread message.
    import threading

    lib = _native.lib()
    stop = threading.Event()
    errors = []

    def setter():
        i = 0
        while not stop.is_set():
            lib.fa_set_max_splits(i % 5)
            lib.fa_set_wait_limit_ns((i % 3) * 1_000_000)
            i += 1

    def caller():
        try:
            for _ in range(20000):
                if lib.fa_fwd_sm100(None, None, None, None, -1, 1, 128, 0, 0.125, None) != -1:
                    errors.append("negative size accepted")
                if "negative" not in _native.last_error():
                    errors.append(_native.last_error())
                if lib.fa_fwd_sm100(8, 16, 32, 48, 1, 1, 128, 0, 0.125, None) != -1:
                    errors.append("misaligned pointer accepted")
        finally:
            stop.set()

    threads = [threading.Thread(target=setter), threading.Thread(target=caller)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=120)
    lib.fa_set_max_splits(0)
    lib.fa_set_wait_limit_ns(0)
    assert not errors, errors[:3]


def test_training_entry_points_validate_without_gpu():
    lib = _native.lib()
    assert lib.fa_bwd_sm100(None, None, None, None, None, None, None, None, None, 0, 4, 128, 0,
                            0.125, None) == 0
    assert lib.fa_bwd_sm100(None, None, None, None, None, None, None, None, None, 1, 1, 128, 0,
                            0.125, None) == -1
    assert "null" in _native.last_error()
    args9 = [None] * 9
    assert lib.fa_bwd_sm100_varlen(*args9, 1, 1, -1, 128, 0, 0.125, None) == -1
    assert "negative" in _native.last_error()
    assert lib.fa_bwd_sm100_varlen(*args9, 0, 1, 128, 256, 0, 0.125, None) == 0
    assert lib.fa_bwd_sm100_varlen(*args9, 1, 1, 128, 256, 0, 0.125, None) == -1
    assert "null" in _native.last_error()
    aligned, odd = [4096] * 9, [4096] * 8 + [4104]
    assert lib.fa_bwd_sm100_varlen(*odd, 1, 1, 128, 256, 0, 0.125, None) == -1
    assert "16-byte aligned" in _native.last_error()
    assert lib.fa_bwd_sm100_varlen(*aligned, 1, 1, 128, 256, 0, 0.0, None) == -1
    assert "scale" in _native.last_error()
    assert lib.fa_bwd_sm100_varlen(*aligned, 1, 1, 128, 0, 0, 0.125, None) == -1
    assert "key length" in _native.last_error()
    assert lib.fa_bwd_sm100_varlen(*aligned, 1, 1, 1 << 31, 128, 0, 0.125, None) == -1
    assert "too large" in _native.last_error()
    assert lib.fa_fwd_sm100_lse(16, 16, 16, 16, None, 1, 1, 128, 128, 0, 0.125, None) == -1
    ext = _native.ext()
    x = torch.zeros(1, 1, 128, 64, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="query must be a CUDA tensor"):
        ext.attention_forward_lse(x, x, x, False, None)
