"""CPU checks of the C ABI: the library loads, exports every function that
include/mi.h declares, and fails loudly (no CPU fallback) without a GPU."""
import ctypes
import os
import re

import pytest

import metal_infer as mi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    text = open(os.path.join(ROOT, "include", "mi.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = set(re.findall(r"\b(mi_[a-z0-9_]+)\s*\(", text))
    return sorted(n for n in names if not n.startswith("mi_token_callback"))


def test_header_declares_the_binding_list():
    assert sorted(mi.EXPORTS) == declared_functions()


def test_library_exports_every_declared_symbol():
    lib = mi.lib()
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_version_string():
    assert "sm_100a" in mi.version()


def test_no_device_is_a_loud_error():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(mi.CoreError) as e:
        mi.MetalContext(0)
    assert e.value.status == mi.ERR_NO_DEVICE
    assert "no CUDA device" in e.value.message


def test_null_arguments_are_rejected():
    lib = mi.lib()
    assert lib.mi_context_create(ctypes.c_int(0), None) == mi.ERR_INVALID_ARGUMENT
    assert b"NULL" in lib.mi_last_error_message()
    assert lib.mi_qwen3_config_validate(None) == mi.ERR_INVALID_ARGUMENT


def test_config_validation_matches_reference_rules():
    cfg = mi.Qwen3Config.from_dict(mi.QWEN3_0_6B)
    assert mi.lib().mi_qwen3_config_validate(ctypes.byref(cfg)) == mi.OK
    bad = mi.Qwen3Config.from_dict(dict(mi.QWEN3_0_6B, head_dim=127))
    assert mi.lib().mi_qwen3_config_validate(ctypes.byref(bad)) == mi.ERR_CONFIG
    bad = mi.Qwen3Config.from_dict(dict(mi.QWEN3_0_6B, num_key_value_heads=3))
    assert mi.lib().mi_qwen3_config_validate(ctypes.byref(bad)) == mi.ERR_CONFIG
