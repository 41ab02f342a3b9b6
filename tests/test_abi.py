"""CPU-side checks of the C ABI: the library loads, exports every symbol that
include/apt_moe.h declares, and its host-only entry points behave (config
parsing, argument validation).  No compute calls: there is no GPU here."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_symbols():
    text = open(os.path.join(ROOT, "include", "apt_moe.h")).read()
    return re.findall(r"APT_API\s+[\w\s\*]+?\b(apt_moe_\w+)\s*\(", text)


@pytest.fixture(scope="module")
def L():
    from apertura_b200 import build
    build.build()
    from apertura_b200._lib import lib
    return lib()


def test_header_declares_expected(L):
    from apertura_b200._lib import EXPORTED
    assert sorted(header_symbols()) == sorted(EXPORTED)


def test_library_exports_every_header_symbol(L):
    for name in header_symbols():
        assert hasattr(L, name), name


def test_version(L):
    assert b"sm_100a" in L.apt_moe_version()


def test_config_from_json_text_config(L):
    from apertura_b200 import ESModelConfig
    text = ('{"architectures": ["Gemma4ForConditionalGeneration"], "hidden_size": 1, '
            '"text_config": {"hidden_size": 2816, "num_experts": 128, "top_k_experts": 8, '
            '"moe_intermediate_size": 704, "enable_moe_block": true, "rms_norm_eps": 1e-06, '
            '"nested": {"hidden_size": 3}}}')
    c = ESModelConfig.from_config_json(text)
    assert (c.hidden_size, c.num_experts, c.top_k_experts, c.moe_intermediate_size) == (
        2816, 128, 8, 704)
    assert c.enable_moe_block and abs(c.rms_norm_eps - 1e-6) < 1e-12
    # runtime knobs keep the reference defaults
    assert (c.moe_sparse, c.quant_bits, c.quant_group_size) == (False, 0, 64)


def test_config_from_json_flat(L):
    from apertura_b200 import ESModelConfig
    c = ESModelConfig.from_config_json('{"hidden_size": 64, "num_experts": 16, '
                                       '"top_k_experts": 4, "moe_intermediate_size": 64}',
                                       moe_sparse=True)
    assert (c.hidden_size, c.num_experts, c.top_k_experts, c.moe_intermediate_size) == (
        64, 16, 4, 64)
    assert c.moe_sparse


def test_create_rejects_bad_config(L):
    from apertura_b200._lib import AptMoeConfig
    h = ctypes.c_void_p()
    for bad in [dict(hidden_size=100), dict(top_k_experts=0), dict(quant_bits=3),
                dict(num_experts=4, top_k_experts=8)]:
        c = dict(hidden_size=2816, num_experts=128, top_k_experts=8, moe_intermediate_size=704,
                 rms_norm_eps=1e-6, enable_moe_block=1, moe_sparse=1, quant_bits=0,
                 quant_group_size=64, max_tokens=16, device=0)
        c.update(bad)
        cfg = AptMoeConfig(**c)
        assert L.apt_moe_create(ctypes.byref(cfg), ctypes.byref(h)) in (1, 2)


def test_null_arguments(L):
    assert L.apt_moe_config_from_json(None, None) == 1
    assert L.apt_moe_create(None, None) == 1
    assert L.apt_moe_destroy(None) == 0
    assert L.apt_moe_route(None, None, 0, None, None, None) == 1


def test_route_noalloc_rejects_misaligned_pointer(L):
    """A pointer off the 16-byte grid is refused before anything is launched
    (the values are never dereferenced: validation runs on the host only)."""
    good, odd = ctypes.c_void_p(0x10000), ctypes.c_void_p(0x10002)
    for x, proj, scale in ((odd, good, good), (good, odd, good), (good, good, odd)):
        st = L.apt_moe_route_noalloc(x, 16, proj, scale, good, 2816, 128, 8, 1e-6, good, good,
                                     None)
        assert st == 1  # APT_ERR_INVALID
