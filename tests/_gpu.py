"""Helpers shared by the GPU tests: torch tensors <-> C-ABI pointers."""
import ctypes

import numpy as np
import torch

from ennx_b200 import _abi


def ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def dev_u16(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, np.uint16).view(np.int16)).cuda()


def host_u16(t: torch.Tensor) -> np.ndarray:
    return t.cpu().numpy().view(np.uint16)


def bf16_dev(a: np.ndarray) -> torch.Tensor:
    """float array -> device bf16 tensor (RNE)."""
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda().to(torch.bfloat16)


def leaves_arr(leaves):
    return (_abi.DenseLeaf * len(leaves))(*[_abi.DenseLeaf(k, o, n, s) for k, o, n, s in leaves])


def terms_arr(terms):
    return (_abi.DenseTerm * len(terms))(*[_abi.DenseTerm(s, c) for s, c in terms])
