"""Thin torch-facing wrappers over the C ABI: allocate outputs and workspaces with torch, pass raw
pointers and the current stream, check the status. No computation happens in Python."""

from __future__ import annotations

import torch

from orthrus_training_b200 import _lib as L


def _require_cuda(*tensors):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise ValueError("orthrus_training_b200 ops run on CUDA tensors only (no CPU fallback)")


def _workspace(nbytes: int, device) -> torch.Tensor | None:
    if nbytes == 0:
        return None
    return torch.empty(int(nbytes), dtype=torch.uint8, device=device)


def gemm(a: torch.Tensor, b: torch.Tensor, *, b_kn: bool = False, out_dtype=None,
         out: torch.Tensor | None = None) -> torch.Tensor:
    """a [M, K] @ (b [N, K])^T (or a @ b for b [K, N] with b_kn). bf16 inputs run on tcgen05 tensor
    cores, fp32 inputs on the exact CUDA-core kernel; fp32 accumulation either way."""
    _require_cuda(a, b)
    if a.dim() != 2 or b.dim() != 2 or a.stride(1) != 1 or b.stride(1) != 1:
        raise ValueError("gemm takes row-major 2-D operands")
    M, K = a.shape
    N = b.shape[1] if b_kn else b.shape[0]
    if (b.shape[0] if b_kn else b.shape[1]) != K:
        raise ValueError(f"gemm shape mismatch {tuple(a.shape)} x {tuple(b.shape)}")
    lib = L.lib()
    stream = L.stream_of(a.device)
    if a.dtype == torch.bfloat16 and b.dtype == torch.bfloat16:
        out_dtype = out_dtype or torch.bfloat16
        c = out if out is not None else torch.empty(M, N, dtype=out_dtype, device=a.device)
        ws = _workspace(lib.orthrus_gemm_workspace_bytes(M, N, K), a.device)
        L.check(lib.orthrus_gemm_bf16(a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0),
                                      c.data_ptr(), c.stride(0), M, N, K, int(b_kn),
                                      int(c.dtype == torch.float32), L.ptr(ws),
                                      0 if ws is None else ws.numel(), stream), "gemm_bf16")
        return c
    if b_kn:
        raise ValueError("the CUDA-core gemm takes b as [N, K]")
    code = L.dtype_code(a.dtype)
    c = out if out is not None else torch.empty(M, N, dtype=a.dtype, device=a.device)
    ws = _workspace(lib.orthrus_gemm_simt_workspace_bytes(M, N, K), a.device)
    L.check(lib.orthrus_gemm_simt(a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0),
                                  c.data_ptr(), c.stride(0), M, N, K, code, L.ptr(ws),
                                  0 if ws is None else ws.numel(), stream), "gemm_simt")
    return c


def lmhead_kl(student, teacher, index, weight, row_weight=None, offsets=None, num_offsets=0,
              need_grad=True, chunk_rows=4096):
    """Fused LM head + log-softmax + KL(teacher || student) (FusedLinearForwardKL.forward math).
    Returns (total fp32 [], kl_rows fp32 [n], agree bool [n], grad [n, d] or None,
    kl_by_offset fp32 [num_offsets] or None, agree_by_offset int64 [num_offsets] or None)."""
    _require_cuda(student, teacher, index, weight, row_weight, offsets)
    dt = student.dtype
    code = L.dtype_code(dt)
    if teacher.dtype != dt or weight.dtype != dt:
        raise ValueError("student, teacher and weight must share a dtype")
    student, teacher, weight = student.contiguous(), teacher.contiguous(), weight.contiguous()
    index = index.to(torch.int64).contiguous()
    n, d = student.shape
    m = teacher.shape[0]
    V = weight.shape[0]
    dev = student.device
    pad = (-d) % 64 if dt == torch.bfloat16 else 0
    if pad:  # the tensor-core path consumes the hidden dimension in 64-wide k-blocks
        student = torch.nn.functional.pad(student, (0, pad))
        teacher = torch.nn.functional.pad(teacher, (0, pad))
        weight = torch.nn.functional.pad(weight, (0, pad))
    dp = d + pad
    lib = L.lib()
    total = torch.empty((), dtype=torch.float32, device=dev)
    kl_rows = torch.empty(n, dtype=torch.float32, device=dev)
    agree = torch.empty(n, dtype=torch.uint8, device=dev)
    grad = torch.empty(n, dp, dtype=dt, device=dev) if need_grad else None
    kbo = abo = None
    if offsets is not None:
        offsets = offsets.to(torch.int64).contiguous()
        kbo = torch.empty(num_offsets, dtype=torch.float32, device=dev)
        abo = torch.empty(num_offsets, dtype=torch.int64, device=dev)
    if row_weight is not None:
        row_weight = row_weight.to(torch.float32).contiguous()
    nbytes = lib.orthrus_lmhead_kl_workspace_bytes(n, m, V, dp, chunk_rows, code)
    ws = torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=dev)
    L.check(lib.orthrus_lmhead_kl_fwd(
        L.ptr(student), n, L.ptr(teacher), m, L.ptr(index), L.ptr(weight), V, dp, L.ptr(row_weight),
        L.ptr(offsets), int(num_offsets), L.ptr(total), L.ptr(kl_rows), L.ptr(agree), L.ptr(grad),
        L.ptr(kbo), L.ptr(abo), chunk_rows, L.ptr(ws), ws.numel(), code, L.stream_of(dev)),
        "lmhead_kl_fwd")
    if grad is not None and pad:
        grad = grad[:, :d]
    return total, kl_rows, agree.bool(), grad, kbo, abo


def lmhead_kl_backward(grad: torch.Tensor, grad_total: torch.Tensor) -> torch.Tensor:
    """grad * grad_total, as FusedLinearForwardKL.backward."""
    _require_cuda(grad, grad_total)
    grad = grad.contiguous()
    out = torch.empty_like(grad)
    gt = grad_total.to(torch.float32).reshape(1).contiguous()
    L.check(L.lib().orthrus_lmhead_kl_bwd(grad.data_ptr(), gt.data_ptr(), out.data_ptr(),
                                          grad.numel(), L.dtype_code(grad.dtype),
                                          L.stream_of(grad.device)), "lmhead_kl_bwd")
    return out
