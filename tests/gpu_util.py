"""Helpers shared by the GPU tests: numpy <-> CUDA tensors (bf16 carried as uint16 bits) and the
tolerances the parity claims use."""

import numpy as np
import torch

FP32_REL = 1e-5   # fp32 attention: max|got - want| / max|want|
BF16_ABS = 2e-2   # bf16/fp16 attention: max-abs error against the fp32 oracle


def to_cuda(arr, dtype=None):
    a = np.asarray(arr)
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16).cuda()
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t.to(dtype) if dtype is not None else t


def to_numpy(t: torch.Tensor) -> np.ndarray:
    t = t.detach().contiguous().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    if t.dtype == torch.float16:
        return t.float().numpy()
    return t.numpy()


def as_f64(t) -> np.ndarray:
    from oracle.paged_oracle import as_float

    if isinstance(t, torch.Tensor):
        t = to_numpy(t)
    return as_float(t, np.float64)


def assert_attention_close(got, want, dtype: str):
    g, w = as_f64(got), as_f64(want)
    err = np.abs(g - w).max()
    if dtype == "float32":
        scale = max(np.abs(w).max(), 1e-30)
        assert err / scale <= FP32_REL, f"fp32 relative error {err / scale:.3e} > {FP32_REL}"
    else:
        assert err <= BF16_ABS, f"{dtype} max-abs error {err:.3e} > {BF16_ABS}"
    return err
