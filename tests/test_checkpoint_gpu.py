"""Quantized checkpoints (ltm_block_save / _load, the bank alone with
ltm_block_save_memory / _load_memory): a block restored from a file gives
bit-identical outputs without its fp32 master weights, the bank written by a
forward survives the round trip, and damaged or mismatched files are refused
with LTM_ERR_INVALID_ARG (checksums, dimensions, scheme, kind) without
touching the block."""
import numpy as np
import pytest

from _util import as_f32, to_device
from test_block_gpu import make

pytestmark = pytest.mark.gpu

SCHEMES = [("w8a8", "f16"), ("w8a8", "bf16"), ("w4a16", "bf16"), ("w8a32", "f32")]


def _block(ltm, scheme, dt, seed, memory_write=False, H=256, F=512, Ms=64, **kw):
    from ltm_b200 import synthetic
    cfg, q, ocfg = make(ltm, scheme, dt, H, 4, F, Ms, memory_write=memory_write, **kw)
    blk = ltm.TitanBlock(cfg, q)
    blk.load_weights(synthetic.block_weights(H, F, Ms, seed))
    return blk, cfg, q


@pytest.mark.parametrize("scheme,dt", SCHEMES)
def test_checkpoint_round_trip_is_bit_exact(ltm, tmp_path, scheme, dt):
    from ltm_b200 import synthetic
    blk, cfg, q = _block(ltm, scheme, dt, 3, memory_write=True)
    x = to_device(synthetic.activations(2 * 48, 256, 4), dt).reshape(2, 48, 256)
    blk(x)  # writes the bank
    path = tmp_path / "block.ltm"
    blk.save(path)
    saved_bank = as_f32(blk.memory())
    y_ref = as_f32(blk(x))
    mem_ref = as_f32(blk.memory())
    fresh = ltm.TitanBlock(cfg, q)  # no fp32 weights: everything from the file
    fresh.load(path)
    assert np.array_equal(as_f32(fresh.memory()), saved_bank), "restored bank differs"
    y = as_f32(fresh(x))
    assert np.array_equal(y, y_ref), "restored block differs"
    # the write's column sums of g * x accumulate with atomics in no fixed
    # order, so the next write agrees to rounding (an ulp of the bank dtype)
    atol = 1e-6 if dt == "f32" else 4e-3
    assert np.abs(as_f32(fresh.memory()) - mem_ref).max() <= atol, "bank after the next write"
    assert ltm.device_error() == 0
    blk.close()
    fresh.close()


def test_bank_alone_round_trip(ltm, tmp_path):
    from ltm_b200 import synthetic
    blk, cfg, q = _block(ltm, "w8a8", "bf16", 5, memory_write=True)
    x = to_device(synthetic.activations(64, 256, 6), "bf16").reshape(1, 64, 256)
    blk(x)
    written = as_f32(blk.memory())
    blk.save_memory(tmp_path / "bank.ltm")
    other, _, _ = _block(ltm, "w8a8", "bf16", 5)  # same weights, pristine bank
    assert not np.array_equal(as_f32(other.memory()), written)
    other.load_memory(tmp_path / "bank.ltm")
    assert np.array_equal(as_f32(other.memory()), written)
    # the next forward reads the loaded bank (K_M | V_M recomputed from it)
    y1 = as_f32(blk(x))
    y2 = as_f32(other(x))
    assert np.array_equal(y1, y2)
    blk.close()
    other.close()


def test_damaged_and_mismatched_checkpoints_are_refused(ltm, tmp_path):
    blk, cfg, q = _block(ltm, "w8a8", "f16", 7)
    path = tmp_path / "b.ltm"
    blk.save(path)
    data = bytearray(path.read_bytes())

    def refused(raw, target, fn="load"):
        p = tmp_path / "x.ltm"
        p.write_bytes(bytes(raw))
        with pytest.raises(ltm.LtmError) as e:
            getattr(target, fn)(p)
        assert e.value.status == ltm.ERR_INVALID_ARG
        return str(e.value)

    flipped = bytearray(data)
    flipped[-40] ^= 0x10  # inside the last section (the bank)
    assert "checksum" in refused(flipped, blk)
    assert "truncated" in refused(data[: len(data) // 2], blk)
    hdr = bytearray(data)
    hdr[10] ^= 1  # the version field
    assert "version" in refused(hdr, blk) or "checksum" in refused(hdr, blk)
    other_dims, _, _ = _block(ltm, "w8a8", "f16", 7, F=1024)
    assert "dimensions" in refused(data, other_dims)
    other_scheme, _, _ = _block(ltm, "w4a16", "f16", 7)
    assert "scheme" in refused(data, other_scheme)
    bank = tmp_path / "bank.ltm"
    blk.save_memory(bank)
    assert "bank" in refused(bank.read_bytes(), blk)
    assert "block" in refused(data, blk, "load_memory")
    # a file damaged in its last section leaves a block with other weights as
    # it was: every section is checked before the first one is copied
    from ltm_b200 import synthetic
    x = to_device(synthetic.activations(32, 256, 8), "f16").reshape(1, 32, 256)
    keep, _, _ = _block(ltm, "w8a8", "f16", 11)
    y_before = as_f32(keep(x))
    refused(flipped, keep)
    assert np.array_equal(as_f32(keep(x)), y_before), "a refused load changed the block"
    for b in (blk, other_dims, other_scheme, keep):
        b.close()
