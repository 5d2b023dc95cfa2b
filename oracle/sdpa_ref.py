"""The reference's attention call restated for CPU use as a checker and a timed baseline.

TEST / BASELINE INFRASTRUCTURE ONLY (tests/, __graft_entry__.smoke(), bench.py's CPU legs).

harness/sp_runtime.py:119-121 runs
    with sdpa_kernel([SDPBackend.FLASH_ATTENTION]):
        oh = torch.nn.functional.scaled_dot_product_attention(qh, kh, vh)
on [1, H/W, S, 128] tensors, non-causal, default scale 1/sqrt(128). This module makes the
same call (PyTorch's CPU flash kernel when the tensors live on the host).
"""
import torch
from torch.nn.attention import SDPBackend, sdpa_kernel


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    with sdpa_kernel([SDPBackend.FLASH_ATTENTION]):
        return torch.nn.functional.scaled_dot_product_attention(q, k, v)
