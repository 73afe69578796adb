"""Mixture-of-experts block (Mixtral): router, top-k, expert-grouped GEMMs,
weighted combine; expert parallel across tensor-parallel ranks.

With the residual stream replicated on every rank, expert parallelism needs
no token all-to-all: each rank routes all tokens, runs only its E/n local
experts on the rows routed to them (one grouped tcgen05 GEMM per
projection, expert row offsets stay on the device), combines them per token
with the routing weights, and the cross-rank sum is the same fused NVLink
reduction used after the row-parallel projections (``tp.reduce``), written
straight from the combine into the symmetric buffer.

Parity: crates/swiftllm-models/src/layers/mlp.rs:207-258 (MoeMlp: router ->
top-k -> route -> combine; a zero-returning placeholder in the reference).
Routing follows Mixtral: softmax over experts, top-k, renormalise.
"""

from __future__ import annotations

import torch

from .. import ops
from ..ops import reference as ref


def moe_forward(model, L, x: torch.Tensor) -> torch.Tensor:
    c = model.cfg
    k = c.num_experts_per_tok
    T, H = x.shape
    if not x.is_cuda:
        logits = ref.linear(x, L.router).float()
        w, ids = ref.moe_topk_softmax(logits, k)
        out = torch.zeros(T, H, dtype=torch.float32)
        for le in range(model.e_local):
            rows, slot = (ids == model.e0 + le).nonzero(as_tuple=True)
            if rows.numel() == 0:
                continue
            h = ref.silu_and_mul(ref.linear(x[rows], L.w13[le]))
            y = ref.linear(h, L.w2[le]).float()
            out.index_add_(0, rows, y * w[rows, slot].unsqueeze(1))
        return out.to(x.dtype)
    C = ops.cuda_ext()
    logits = ops.linear(x, L.router).float()
    w = torch.empty(T, k, dtype=torch.float32, device=x.device)
    ids = torch.empty(T, k, dtype=torch.int32, device=x.device)
    C.moe_route(logits, k, True, w, ids)
    El = model.e_local
    offsets = torch.empty(El + 1, dtype=torch.int32, device=x.device)
    perm = torch.empty(T * k, dtype=torch.int32, device=x.device)
    inv = torch.empty(T * k, dtype=torch.int32, device=x.device)
    C.moe_permute(ids, model.e0, El, offsets, perm, inv)
    xg = torch.empty(T * k, H, dtype=x.dtype, device=x.device)
    C.moe_gather(xg, x, perm)
    ops._count(3)
    avg = max(1, (T * k) // max(c.num_experts, 1))
    I2 = L.w13.shape[1]
    h = torch.empty(T * k, I2, dtype=x.dtype, device=x.device)
    ops._count(C.gemm_grouped(h, xg, L.w13, offsets, avg))
    a = ops.silu_and_mul(h)
    y = torch.empty(T * k, H, dtype=x.dtype, device=x.device)
    ops._count(C.gemm_grouped(y, a, L.w2, offsets, avg))
    out = model._reduce_slot(T)
    if out is None:
        out = torch.empty(T, H, dtype=x.dtype, device=x.device)
    C.moe_combine(out, y, w, inv)
    ops._count()
    return out
