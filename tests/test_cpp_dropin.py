"""The C++ drop-in header (include/ltm/titan_block.hpp) on the CPU: the GPU
test program that uses it compiles, and the pybind shim that re-points the
reference's `_ltm` module at this library compiles, imports
and exposes TitanBlockConfig with the reference's defaults."""
import importlib.util
import sys
from pathlib import Path

import pytest

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE / "cpp"))


def test_titan_block_test_program_compiles():
    import cpp_build
    exe = cpp_build.build_test()
    assert exe.exists()


def test_pybind_shim_compiles_and_imports():
    import cpp_build
    pytest.importorskip("pybind11")
    mod_path = cpp_build.build_pybind_shim()
    spec = importlib.util.spec_from_file_location("ltm_pybind_shim", mod_path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    c = mod.TitanBlockConfig()
    assert (c.hidden_dim, c.ffn_dim, c.num_heads, c.head_dim, c.memory_slots) == (768, 3072, 12,
                                                                                   64, 512)
    assert abs(c.memory_update_rate - 0.9) < 1e-7 and c.use_rotary == 1 and c.use_alibi == 0
    c.hidden_dim = 256
    assert c.hidden_dim == 256
    assert hasattr(mod, "TitanModelImpl")
