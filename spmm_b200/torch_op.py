"""torch custom op for GCN / GraphSAGE aggregation: ``torch.ops.tcaspmm.spmm``.

    Y = torch.ops.tcaspmm.spmm(crow, col, val, X)      # Y = A @ X, fp32, shape (M, N)

``crow`` (int32/int64, M+1), ``col`` (int32/int64, nnz) and ``val`` (nnz) describe A in
CSR on the host or on X's device; ``X`` is a CUDA tensor (K x N, float32 / float16 /
bfloat16; float32 X uses the TF32 tensor-core path when
``torch.backends.cuda.matmul.allow_tf32`` is set, as PyTorch's own matmuls do).  The op runs tcaspmm's plan-based C-ABI path (``spmm_b200/lib/libtcaspmm.so``)
on X's current stream: a plan (host preprocessing + one upload of A) is built the
first time a given (A, N, dtype, device) is seen and reused afterwards, so a GNN layer
pays the preprocessing once per graph.  The gradient with respect to X is
``A^T @ dY``, computed with a second cached plan over the transpose of A; A's values
are treated as constants (the graph does not train).

    Y = torch.ops.tcaspmm.spmm_fused(crow, col, val, X, row_scale, bias, relu, out_dtype)

applies the plan's fused epilogue (row scale, bias, ReLU, fp32/fp16/bf16 output) in
the same kernels; its backward gives dX (through A^T) and d(bias).  There is no CPU or
PyTorch fallback: without the library or a CUDA device the ops raise.
"""
from __future__ import annotations

from typing import Dict, Optional, Tuple

import numpy as np
import torch

from . import CSR, Epilogue, Plan, as_dtype


class _Entry:
    """A cached plan and the CSR tensors it was built from.

    The entry keeps those tensors alive, so their memory cannot be handed to a new
    graph while the plan is cached, and it is reused only for the very same tensor
    objects at the same versions: an in-place edit of crow, col or val (which bumps
    the tensor's version counter) or a different tensor at a recycled address both
    build a new plan."""

    __slots__ = ("plan", "tensors", "versions")

    def __init__(self, plan: Plan, tensors: Tuple[torch.Tensor, ...]):
        self.plan = plan
        self.tensors = tensors
        self.versions = tuple(t._version for t in tensors)

    def matches(self, tensors: Tuple[torch.Tensor, ...]) -> bool:
        return all(a is b for a, b in zip(self.tensors, tensors)) and \
            self.versions == tuple(t._version for t in tensors)


_PLANS: Dict[Tuple, _Entry] = {}
_MAX_PLANS = 16


def _key(crow: torch.Tensor, col: torch.Tensor, val: torch.Tensor, N: int, dt, dev: int, transposed: bool) -> Tuple:
    return (crow.data_ptr(), col.data_ptr(), val.data_ptr(), tuple(crow.shape), tuple(col.shape), crow.device.type,
            int(N), dt.name, dev, transposed)


def _host_csr(crow: torch.Tensor, col: torch.Tensor, val: torch.Tensor, ncol: int, transposed: bool) -> CSR:
    rp = crow.detach().to("cpu", torch.int64).numpy()
    ci = col.detach().to("cpu", torch.int64).numpy()
    va = val.detach().to("cpu", torch.float32).numpy()
    M = rp.shape[0] - 1
    if not transposed:
        return CSR(M, ncol, rp, ci.astype(np.int32), va)
    # CSR of A^T: stable sort of the nonzeros by column keeps rows ascending.
    rows = np.repeat(np.arange(M, dtype=np.int64), np.diff(rp))
    order = np.argsort(ci, kind="stable")
    trp = np.zeros(ncol + 1, np.int64)
    np.add.at(trp, ci + 1, 1)
    return CSR(ncol, M, np.cumsum(trp), rows[order].astype(np.int32), va[order])


def _plan(crow, col, val, ncol: int, X: torch.Tensor, transposed: bool) -> Plan:
    dt = as_dtype(X.dtype)
    if dt == as_dtype("f32") and torch.backends.cuda.matmul.allow_tf32:
        dt = as_dtype("tf32")  # PyTorch's TF32 switch: fp32 X through the TF32 tensor-core windows
    dev = X.device.index if X.device.index is not None else torch.cuda.current_device()
    k = _key(crow, col, val, X.shape[1], dt, dev, transposed)
    tensors = (crow, col, val)
    e = _PLANS.get(k)
    if e is not None and not e.matches(tensors):
        _PLANS.pop(k).plan.close()  # same addresses and shapes, different or edited tensors
        e = None
    if e is None:
        if len(_PLANS) >= _MAX_PLANS:
            _PLANS.pop(next(iter(_PLANS))).plan.close()
        e = _Entry(Plan(_host_csr(crow, col, val, ncol, transposed), X.shape[1], dt, 1, [dev]), tensors)
        _PLANS[k] = e
    return e.plan


def clear_plan_cache() -> None:
    while _PLANS:
        _PLANS.popitem()[1].plan.close()


@torch.library.custom_op("tcaspmm::spmm", mutates_args=())
def spmm(crow: torch.Tensor, col: torch.Tensor, val: torch.Tensor, X: torch.Tensor) -> torch.Tensor:
    if not X.is_cuda:
        raise ValueError("tcaspmm::spmm needs X on a CUDA device")
    X = X.contiguous()
    M = crow.shape[0] - 1
    p = _plan(crow, col, val, X.shape[0], X, transposed=False)
    out = torch.empty((M, X.shape[1]), device=X.device, dtype=torch.float32)
    p.execute1(X, out, torch.cuda.current_stream(X.device))
    return out


@spmm.register_fake
def _(crow, col, val, X):
    return X.new_empty((crow.shape[0] - 1, X.shape[1]), dtype=torch.float32)


@torch.library.custom_op("tcaspmm::spmm_t", mutates_args=())
def spmm_t(crow: torch.Tensor, col: torch.Tensor, val: torch.Tensor, dY: torch.Tensor, ncol: int) -> torch.Tensor:
    """A^T @ dY for the backward pass (A given in CSR with ncol columns)."""
    dY = dY.contiguous()
    p = _plan(crow, col, val, ncol, dY, transposed=True)
    out = torch.empty((ncol, dY.shape[1]), device=dY.device, dtype=torch.float32)
    p.execute1(dY, out, torch.cuda.current_stream(dY.device))
    return out


@spmm_t.register_fake
def _(crow, col, val, dY, ncol):
    return dY.new_empty((ncol, dY.shape[1]), dtype=torch.float32)


def _setup(ctx, inputs, output):
    crow, col, val, X = inputs
    ctx.save_for_backward(crow, col, val)
    ctx.ncol = X.shape[0]
    ctx.x_dtype = X.dtype


def _backward(ctx, grad):
    crow, col, val = ctx.saved_tensors
    g = grad.to(ctx.x_dtype) if ctx.x_dtype != torch.float32 else grad
    dX = torch.ops.tcaspmm.spmm_t(crow, col, val, g, ctx.ncol)
    return None, None, None, dX.to(ctx.x_dtype)


spmm.register_autograd(_backward, setup_context=_setup)


_OUT = {torch.float32: "f32", torch.float16: "f16", torch.bfloat16: "bf16"}


@torch.library.custom_op("tcaspmm::spmm_fused", mutates_args=())
def spmm_fused(crow: torch.Tensor, col: torch.Tensor, val: torch.Tensor, X: torch.Tensor,
               row_scale: Optional[torch.Tensor], bias: Optional[torch.Tensor], relu: bool,
               out_dtype: torch.dtype) -> torch.Tensor:
    """relu?(row_scale[:, None] * (A @ X) + bias) stored as out_dtype, in one pass (the
    plan's fused epilogue: no separate elementwise kernels, 16-bit C halves C's bytes)."""
    if not X.is_cuda:
        raise ValueError("tcaspmm::spmm_fused needs X on a CUDA device")
    if out_dtype not in _OUT:
        raise ValueError(f"out_dtype must be float32, float16 or bfloat16, not {out_dtype}")
    X = X.contiguous()
    M = crow.shape[0] - 1
    p = _plan(crow, col, val, X.shape[0], X, transposed=False)
    out = torch.empty((M, X.shape[1]), device=X.device, dtype=out_dtype)
    rs = row_scale.to(X.device, torch.float32).contiguous() if row_scale is not None else None
    b = bias.to(X.device, torch.float32).contiguous() if bias is not None else None
    p.execute1(X, out, torch.cuda.current_stream(X.device), epilogue=Epilogue(rs, b, relu, _OUT[out_dtype]))
    return out


@spmm_fused.register_fake
def _(crow, col, val, X, row_scale, bias, relu, out_dtype):
    return X.new_empty((crow.shape[0] - 1, X.shape[1]), dtype=out_dtype)


def _setup_fused(ctx, inputs, output):
    crow, col, val, X, row_scale, bias, relu, out_dtype = inputs
    ctx.save_for_backward(crow, col, val, row_scale, output if relu else None)
    ctx.ncol = X.shape[0]
    ctx.x_dtype = X.dtype
    ctx.has_bias = bias is not None


def _backward_fused(ctx, grad):
    # Y = relu(s * (A X) + b):  dZ = dY * [Y > 0],  dX = A^T (s * dZ),  db = sum_r dZ.
    crow, col, val, row_scale, Y = ctx.saved_tensors
    dZ = grad.float()
    if Y is not None:
        dZ = dZ * (Y > 0)
    db = dZ.sum(0) if ctx.has_bias else None
    if row_scale is not None:
        dZ = dZ * row_scale.to(dZ.device, torch.float32)[:, None]
    dX = torch.ops.tcaspmm.spmm_t(crow, col, val, dZ.to(ctx.x_dtype), ctx.ncol)
    return None, None, None, dX.to(ctx.x_dtype), None, db, None, None


spmm_fused.register_autograd(_backward_fused, setup_context=_setup_fused)


class GCNAggregate(torch.nn.Module):
    """Y = relu?(row_scale * (A_hat @ X) + bias) with a fixed adjacency A_hat in CSR (the GCN /
    GraphSAGE-mean propagation step); without row_scale, bias or relu it is plain A_hat @ X."""

    def __init__(self, crow: torch.Tensor, col: torch.Tensor, val: torch.Tensor,
                 row_scale: Optional[torch.Tensor] = None, bias: Optional[torch.Tensor] = None,
                 relu: bool = False):
        super().__init__()
        self.register_buffer("crow", crow)
        self.register_buffer("col", col)
        self.register_buffer("val", val)
        self.register_buffer("row_scale", row_scale)
        self.bias = bias
        self.relu = relu

    def forward(self, X: torch.Tensor) -> torch.Tensor:
        if self.row_scale is None and self.bias is None and not self.relu:
            return torch.ops.tcaspmm.spmm(self.crow, self.col, self.val, X)
        return torch.ops.tcaspmm.spmm_fused(self.crow, self.col, self.val, X, self.row_scale, self.bias,
                                            self.relu, torch.float32)
