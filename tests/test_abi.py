"""CPU tests of the boundary: libriallm_cuda.so builds for sm_100a, loads,
exports every function include/riallm_cuda.h declares, and the host-side
mirror of the reference API behaves like src/config.rs. No GPU compute."""
import ctypes
import os
import re

import pytest

from conftest import ROOT


def header_functions():
    src = open(os.path.join(ROOT, "include", "riallm_cuda.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(riallm_\w+)\s*\(", src)))


def test_library_exports_every_declared_symbol(rb):
    lib = ctypes.CDLL(rb.LIB_PATH)
    names = header_functions()
    assert len(names) >= 19
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) == set(rb.SIGNATURES), set(names) ^ set(rb.SIGNATURES)


def test_abi_version_and_size_helpers(rb):
    L = rb.lib()
    assert L.riallm_cuda_abi_version() == 1
    assert L.riallm_quant_num_blocks(1, 4097) == 65
    assert L.riallm_quant_data_bytes(1, 4097) == 2049
    assert L.riallm_quant_num_blocks(2, 4097) == 33
    assert L.riallm_quant_data_bytes(2, 4097) == 4097


def test_context_without_gpu_fails_cleanly(rb):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    p = ctypes.c_void_p()
    assert rb.lib().riallm_cuda_ctx_create(0, ctypes.byref(p)) != 0
    assert not p.value


def test_compression_type_from_str(rb):
    """tests/integration_test.rs:63-79."""
    C = rb.CompressionType
    assert C.from_str("4bit") == C.FourBit
    assert C.from_str("8bit") == C.EightBit
    assert C.from_str("none") == C.None_ and C.from_str("") == C.None_
    with pytest.raises(rb.ConfigError):
        C.from_str("invalid")


def test_model_options_defaults(rb):
    """src/config.rs:399-411 and tests/integration_test.rs:81-89."""
    o = rb.ModelOptions()
    assert o.compression == rb.CompressionType.None_
    assert o.device.is_cuda() and o.device.device_id() == 0
    assert o.prefetch_layers and o.prefetch_buffer_size == 2
    assert o.dtype == "float16" and o.max_seq_len is None and not o.profiling_mode

