"""Helpers shared by the GPU tests."""
import numpy as np
import torch


def to_dev_bf16(u16: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(u16).view(np.int16)).view(torch.bfloat16).cuda()


def bits(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    if t.dtype == torch.float8_e4m3fn:
        return t.view(torch.uint8).numpy()
    return t.numpy()


def rand_bf16(rows, cols, seed, outliers=True, kind="normal"):
    g = torch.Generator().manual_seed(seed)
    if kind == "student_t":
        z = torch.randn(rows, cols, generator=g)
        chi = torch.distributions.Chi2(torch.tensor(4.0)).sample((rows, 1))
        w = 0.02 * z / torch.sqrt(chi / 4.0)
    else:
        w = 0.02 * torch.randn(rows, cols, generator=g)
    if outliers:
        m = torch.rand(rows, cols, generator=g) < 0.001
        w = torch.where(m, w * 50, w)
    if rows >= 3:
        w[0] = 0
        w[2] *= 1e-6
    return w.to(torch.bfloat16)


def np_f32(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()
