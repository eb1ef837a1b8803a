"""LinearMoE with the reference's constructor and parameters (one/linear_moe.py:6-114); its
forward runs the native router + shared Linear (C ABI one_linear_moe): gate, softmax over r,
expert factors, per-expert biased sums, the reference's top-k selection, combine, Linear.
"""
from __future__ import annotations

import ctypes

import torch
from torch import nn

from . import _capi as C


class LinearMoE(nn.Linear):
    def __init__(self, in_features: int, out_features: int, bias: bool = True, device=None, dtype=None,
                 num_experts: int = 1000, r: int = 4, top_k: int = 4):
        super().__init__(in_features, out_features, bias=bias, device=device, dtype=dtype)
        self.num_experts = num_experts
        self.r = r
        self.top_k = min(top_k, num_experts)
        self.gate = nn.Linear(in_features, r, bias=False, device=device, dtype=dtype)
        self.experts = nn.Parameter(torch.ones(num_experts, device=device, dtype=dtype))
        self.bias2 = nn.Parameter(torch.zeros(num_experts, in_features, device=device, dtype=dtype))
        self.activation = nn.SiLU()
        self.eps = 1e-8
        self.reset_parameters()
        self._ws = None
        self.last_indices = None  # top-k experts of the last forward, int32 [N, k]

    def reset_parameters(self) -> None:
        super().reset_parameters()
        if hasattr(self, "gate"):
            nn.init.xavier_uniform_(self.gate.weight, gain=1.0)
        if hasattr(self, "experts"):
            nn.init.normal_(self.experts, mean=0.0, std=0.1)
        if hasattr(self, "bias2"):
            nn.init.zeros_(self.bias2)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if not x.is_cuda:
            raise RuntimeError("LinearMoE runs on the B200 engine: pass CUDA tensors")
        orig = x.shape
        x2 = x.reshape(-1, x.size(-1)).contiguous()
        n, fin = x2.shape
        dt = x2.dtype
        code = C.dtype_code(dt)
        w = self.weight.to(dt).contiguous()
        b = None if self.bias is None else self.bias.to(dt).contiguous()
        g = self.gate.weight.to(dt).contiguous()
        e = self.experts.to(dt).contiguous()
        b2 = self.bias2.to(dt).contiguous()
        out = torch.empty(n, self.out_features, dtype=dt, device=x.device)
        idx = torch.empty(n, self.top_k, dtype=torch.int32, device=x.device)
        need = C.LIB.one_linear_moe_workspace_bytes(n, fin, self.r, code)
        if self._ws is None or self._ws.numel() < need or self._ws.device != x.device:
            self._ws = torch.empty(need, dtype=torch.uint8, device=x.device)
        C.check(C.LIB.one_linear_moe(C.ptr(x2), n, fin, self.out_features, C.ptr(w), C.ptr(b), C.ptr(g), C.ptr(e),
                                     C.ptr(b2), self.num_experts, self.r, self.top_k, code, C.ptr(out), C.ptr(idx),
                                     C.ptr(self._ws), self._ws.numel(),
                                     ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)), "one_linear_moe")
        self.last_indices = idx
        if len(orig) > 2:
            out = out.view(*orig[:-1], -1)
        return out
