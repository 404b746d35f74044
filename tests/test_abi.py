"""The C-ABI library loads and exports every entry point include/ltm_b200.h
declares (no device calls)."""
import ctypes
import re

from conftest import ROOT

HEADER = ROOT / "include" / "ltm_b200.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(ltm_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared_functions()
    for must in ("ltm_quantize_int8_per_channel", "ltm_quantize_int4_grouped",
                 "ltm_linear_w8a8", "ltm_linear_w4a16", "ltm_block_forward", "ltm_model_forward"):
        assert must in names


def test_library_exports_every_declared_symbol():
    import ltm_b200
    lib = ltm_b200.lib()
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, f"missing exports: {missing}"


def test_version_and_error_string_without_device():
    import ltm_b200
    assert "sm_100a" in ltm_b200.version()
    assert isinstance(ltm_b200.lib().ltm_last_error_string(), bytes)


def test_config_mirror_matches_reference_fields():
    """TitanBlockConfig keeps the reference's field names, order and defaults
    (include/core/transformer/titan_inspired_block.cuh:19-50)."""
    import dataclasses
    import ltm_b200
    ref = [("hidden_dim", 768), ("ffn_dim", 3072), ("num_heads", 12), ("head_dim", 64),
           ("memory_slots", 512), ("memory_dim", 64), ("memory_update_rate", 0.9),
           ("use_memory_compression", True), ("memory_compression_ratio", 0.5),
           ("use_flash_attention", True), ("use_alibi", False), ("use_rotary", True),
           ("dropout_prob", 0.1), ("use_parallel_attention", True), ("use_memory_gating", True),
           ("use_layer_norm", True), ("use_bias", True), ("fuse_operations", True),
           ("learn_memory", True), ("learn_compression", True), ("gradient_checkpointing", True)]
    got = [(f.name, f.default) for f in dataclasses.fields(ltm_b200.TitanBlockConfig)]
    assert got == ref
    assert [f[0] for f in ltm_b200.BlockConfigC._fields_] == [r[0] for r in ref]
    c = ltm_b200.BlockConfigC()
    ltm_b200.lib().ltm_block_config_default(ctypes.byref(c))
    for name, val in ref:
        assert abs(float(getattr(c, name)) - float(val)) < 1e-6, name
