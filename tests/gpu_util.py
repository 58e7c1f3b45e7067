"""Helpers for the GPU tests: device buffers (torch allocations used as plain
CUDA memory) and the seeded synthetic model in host memory."""
import numpy as np


def dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    import torch
    torch.cuda.synchronize()
    return t.cpu().numpy()


def empty_f32(n):
    import torch
    return torch.full((n,), float("nan"), dtype=torch.float32, device="cuda")


def oracle_weights(w):
    """Per-layer (data, scales) pairs as the oracle model wants them."""
    return w
