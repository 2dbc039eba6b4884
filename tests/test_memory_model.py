"""Memory accounting (memory_model.py) against the reference's own expected
values (tests/test_memory_model.py of the reference) and, in this container,
against the reference module itself on a grid of arguments."""

import importlib
import os
import sys

import pytest

from conftest import PACKAGE

mm = importlib.import_module(PACKAGE + ".memory_model")


def test_reference_expected_values():
    assert mm.kv_bytes_per_token_gqa(8, 128, 2) == 4096
    assert mm.kv_bytes_per_token_latent(512, 2) == 1024
    assert mm.estimate_total_kv_cache_bytes(28, 4096, 1, 4096) == 469762048
    assert mm.compression_ratio(4096, 1024) == 4.0
    assert mm.kv_bytes_per_token_gqa(8, 128, 2, include_k_and_v=False) == 2048
    assert mm.kv_bytes_per_token_latent(6, 2) < mm.kv_bytes_per_token_gqa(2, 8, 2)


@pytest.mark.parametrize("value", [0, -1])
def test_invalid_inputs_raise(value):
    with pytest.raises(ValueError):
        mm.kv_bytes_per_token_gqa(value, 128, 2)
    with pytest.raises(ValueError):
        mm.estimate_total_kv_cache_bytes(1, value, 1, 4)
    with pytest.raises(TypeError):
        mm.kv_bytes_per_token_latent(2.0, 2)


def test_cli_table_and_report():
    text = mm.estimate(28, 4096, 1, 8, 128, 512, 2)
    assert "469762048" in text and "4.000x" in text and "448.00 MiB" in text
    r = mm.cache_bytes_report(tokens=1048576, kv_heads=1, head_dim=576, latent_dim=576,
                              dtype_bytes=2)
    assert r["latent_bytes"] == 1048576 * 1152


# The reference's python_ref directory, when a checkout is available (set
# PLKV_REFERENCE to the reference project's root).
_REF = os.path.join(os.environ.get("PLKV_REFERENCE", ""), "python_ref")


@pytest.mark.skipif(not os.environ.get("PLKV_REFERENCE") or not os.path.isdir(_REF),
                    reason="PLKV_REFERENCE does not name a reference checkout")
def test_matches_reference_module():
    sys.path.insert(0, _REF)
    try:
        ref = importlib.import_module("latent_paged_attention.memory_model")
    finally:
        sys.path.remove(_REF)
    for kv, d, b in [(1, 1, 1), (8, 128, 2), (2, 64, 4), (32, 96, 1)]:
        assert mm.kv_bytes_per_token_gqa(kv, d, b) == ref.kv_bytes_per_token_gqa(kv, d, b)
        assert mm.kv_bytes_per_token_latent(kv * d, b) == ref.kv_bytes_per_token_latent(kv * d, b)
        assert mm.compression_ratio(kv * d * b * 2, d * b) == ref.compression_ratio(kv * d * b * 2,
                                                                                    d * b)
        assert (mm.estimate_total_kv_cache_bytes(3, 1000 + kv, b, d)
                == ref.estimate_total_kv_cache_bytes(3, 1000 + kv, b, d))
