"""Small helpers for the GPU tests: numpy <-> device tensors, seeded cases."""
import numpy as np


def dev(torch, a):
    """Copy a numpy array to cuda:0 (keeps dtype; uint16 is moved as int16 bits)."""
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16)).cuda()
    return torch.from_numpy(a).cuda()


def host(t):
    return t.detach().cpu().numpy()


def mat_dev(torch, M):
    """(w, s, z) device tensors of a tiny_kernel.data.Int4Matrix."""
    return dev(torch, M.w), dev(torch, M.s), dev(torch, M.z)
