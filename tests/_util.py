"""Helpers shared by the tests (seeded inputs, dtype plumbing)."""
import numpy as np

DT_NAMES = ("f32", "f16", "bf16")


def torch_dtype(name):
    import torch
    return {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}[name]


def orc_dtype(name):
    return {"f32": 0, "f16": 1, "bf16": 2}[name]


def to_device(a: np.ndarray, dt: str):
    """fp32 numpy -> CUDA tensor of dtype dt (round-to-nearest-even)."""
    import torch
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(torch_dtype(dt)).cuda()


def as_f32(t) -> np.ndarray:
    return t.float().cpu().numpy()


def assert_close(got, want, atol, rtol, what=""):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert got.shape == want.shape, (got.shape, want.shape)
    err = np.abs(got - want)
    bound = atol + rtol * np.abs(want)
    bad = err > bound
    if bad.any():
        i = np.unravel_index(np.argmax(err - bound), err.shape)
        raise AssertionError(f"{what}: {bad.sum()} / {bad.size} outside tolerance "
                             f"(atol={atol}, rtol={rtol}); worst at {i}: got {got[i]}, want {want[i]}, "
                             f"max abs err {err.max():.3e}")
