"""Grouped-expert execution of a mixture-of-experts FFN on the sm_100a kernels.

The (token, slot) assignments are laid out expert by expert, each expert's segment padded to a
multiple of 128 rows (padding rows are zero), so that every 128-row tile of the grouped GEMMs
belongs to one expert.  The layout is computed on the device from the router's choices; the
buffers are sized by the upper bound ``round_up(T k, 128) + 128 E`` so the host never waits for
the counts.  Unused tiles are skipped by the GEMM engine (its ``grp_m`` table holds -1 there).

Forward:  x_perm = gather(x)                         (moe.cu)
          h_pre, h = x_perm W_fc[e]^T, relu(.)^2       (grouped GEMM, ReLU^2 epilogue)
          y_perm = h W_proj[e]^T                       (grouped GEMM)
          y = sum_s w[t, s] y_perm[row(t, s)]          (moe.cu combine)
Backward: d_rows = w dy at each row, dw = dy . y_perm  (moe.cu)
          dh_pre = (d_rows W_proj[e]) 2 relu(h_pre)    (grouped GEMM, ReLU^2-backward epilogue)
          dW_proj[e] += d_rows^T h,  dW_fc[e] += dh_pre^T x_perm   (grouped-K GEMMs over each segment)
          dx_perm = dh_pre W_fc[e];  dx = sum_s dx_perm[row(t, s)]
"""
import torch
from torch.autograd import Function

from nexttransformer_b200.ops._ext import ext

EPI_BF16, EPI_F32, EPI_F32_ACC, EPI_BF16_AXPBY, EPI_RELU2, EPI_RELU2_BWD = range(6)
PAD = 128


def plan(choice, num_experts):
    """Row layout of the assignments ``choice`` [T, k] (int): row_of [T k], src_of [P], grp_m
    [P / 128], grp_k [E + 1] (int32, all on the device) and P."""
    T, k = choice.shape
    dev = choice.device
    flat = choice.reshape(-1).long()
    n = flat.numel()
    P = (n + PAD - 1) // PAD * PAD + PAD * num_experts
    counts = torch.bincount(flat, minlength=num_experts)
    padded = (counts + PAD - 1) // PAD * PAD
    end = padded.cumsum(0)
    start = end - padded
    first = counts.cumsum(0) - counts
    order = torch.argsort(flat, stable=True)
    e_sorted = flat[order]
    rows_sorted = start[e_sorted] + torch.arange(n, device=dev) - first[e_sorted]
    row_of = torch.empty(n, dtype=torch.long, device=dev)
    row_of[order] = rows_sorted
    src_of = torch.full((P,), -1, dtype=torch.int32, device=dev)
    src_of[row_of] = (torch.arange(n, device=dev) // k).to(torch.int32)
    tile_row = torch.arange(P // PAD, device=dev) * PAD
    grp_m = torch.searchsorted(end, tile_row, right=True)
    grp_m = torch.where(tile_row < end[-1], grp_m, torch.full_like(grp_m, -1)).to(torch.int32)
    grp_k = torch.cat((end.new_zeros(1), end)).to(torch.int32)
    return dict(row_of=row_of.to(torch.int32), src_of=src_of, grp_m=grp_m, grp_k=grp_k, P=P, counts=counts)


class _GroupedExperts(Function):
    @staticmethod
    def forward(ctx, x, w, w_fc, w_proj, row_of, src_of, grp_m, grp_k, state=None):
        lib = ext()
        T, d = x.shape
        E, F = w_fc.shape[0], w_fc.shape[1]
        P = src_of.numel()
        xb = x.to(torch.bfloat16).contiguous()
        wf = w_fc.to(torch.bfloat16).contiguous()
        wp = w_proj.to(torch.bfloat16).contiguous()
        x_perm = torch.empty(P, d, device=x.device, dtype=torch.bfloat16)
        lib.moe_gather_rows(xb, src_of, x_perm)
        h_pre = torch.empty(P, F, device=x.device, dtype=torch.bfloat16)
        h = torch.empty_like(h_pre)
        lib.gemm_grouped(x_perm, False, wf, False, h, EPI_RELU2, grp_m, False, None, h_pre, 1.0)
        y_perm = torch.empty(P, d, device=x.device, dtype=torch.bfloat16)
        lib.gemm_grouped(h, False, wp, False, y_perm, EPI_BF16, grp_m, False, None, None, 1.0)
        wf32 = w.float().contiguous()
        out = torch.empty(T, d, device=x.device, dtype=torch.bfloat16)
        lib.moe_combine(y_perm, row_of, wf32, None, out)
        ctx.save_for_backward(x_perm, h_pre, h, y_perm, wf, wp, row_of, grp_m, grp_k, wf32)
        ctx.dtypes = (x.dtype, w.dtype, w_fc.dtype, w_proj.dtype)
        ctx.state = state
        return out.to(x.dtype)

    @staticmethod
    def backward(ctx, dout):
        lib = ext()
        x_perm, h_pre, h, y_perm, wf, wp, row_of, grp_m, grp_k, wf32 = ctx.saved_tensors
        T = dout.shape[0]
        P, d = x_perm.shape
        E, F = wf.shape[0], wf.shape[1]
        dy = dout.to(torch.bfloat16).contiguous()
        d_rows = torch.zeros(P, d, device=dy.device, dtype=torch.bfloat16)
        dw = torch.empty_like(wf32)
        lib.moe_combine_bwd(dy, y_perm, row_of, wf32, d_rows, dw)
        dh_pre = torch.empty(P, F, device=dy.device, dtype=torch.bfloat16)
        lib.gemm_grouped(d_rows, False, wp, True, dh_pre, EPI_RELU2_BWD, grp_m, False, h_pre, None, 1.0)
        state = ctx.state
        # the grouped-K weight-gradient GEMMs accumulate (experts without rows are left untouched):
        # into the experts' main_grad stacks (zeroed once per update) or into fresh zeroed buffers
        dwp = state._g_proj if state is not None else torch.zeros(E, d, F, device=dy.device, dtype=torch.float32)
        lib.gemm_grouped(d_rows, True, h, True, dwp, EPI_F32_ACC, grp_k, True, None, None, 1.0)
        dx_perm = torch.empty(P, d, device=dy.device, dtype=torch.bfloat16)
        lib.gemm_grouped(dh_pre, False, wf, True, dx_perm, EPI_BF16, grp_m, False, None, None, 1.0)
        dwf = state._g_fc if state is not None else torch.zeros(E, F, d, device=dy.device, dtype=torch.float32)
        lib.gemm_grouped(dh_pre, True, x_perm, True, dwf, EPI_F32_ACC, grp_k, True, None, None, 1.0)
        dx = torch.empty(T, d, device=dy.device, dtype=torch.bfloat16)
        lib.moe_combine(dx_perm, row_of, None, None, dx)
        xd, wd, fd, pd = ctx.dtypes
        if state is not None:
            return dx.to(xd), dw.view(T, -1).to(wd), None, None, None, None, None, None, None
        return dx.to(xd), dw.view(T, -1).to(wd), dwf.to(fd), dwp.to(pd), None, None, None, None, None


def fused_route_supported(logits, k):
    E = logits.shape[-1]
    return (logits.is_cuda and E % 32 == 0 and 32 <= E <= 256 and 1 <= k <= min(16, E)
            and getattr(ext(), "moe_route", None) is not None)


class _Route(Function):
    """Router softmax, biased top-k, normalised weights, losses and the row plan (moe_route.cu)."""

    @staticmethod
    def forward(ctx, logits, bias, k, aux_coeff, z_coeff, load):
        choice, w, lse, row_of, src_of, grp_m, grp_k, counts, aux_grad, aux = ext().moe_route(
            logits, bias, k, aux_coeff, z_coeff, load)
        ctx.save_for_backward(logits, lse, choice, w, aux_grad)
        ctx.z = z_coeff
        ctx.mark_non_differentiable(choice, row_of, src_of, grp_m, grp_k, counts)
        return choice, w, aux.sum(), row_of, src_of, grp_m, grp_k, counts

    @staticmethod
    def backward(ctx, _choice, dw, daux, *_plan):
        logits, lse, choice, w, aux_grad = ctx.saved_tensors
        d = ext().moe_route_bwd(logits, lse, choice, w, None if dw is None else dw.float().contiguous(), aux_grad,
                                None if daux is None else daux.float().reshape(1), ctx.z)
        return d, None, None, None, None, None


def fused_route(logits, bias, k, aux_coeff=0.0, z_coeff=0.0, load=None):
    """(choice int32 [T, k], w fp32 [T, k], aux scalar, plan) from fp32 router logits [T, E] in
    three launches; ``plan`` has the keys of ``plan()``.  ``load`` (fp32 [E]) gains the counts."""
    choice, w, aux, row_of, src_of, grp_m, grp_k, counts = _Route.apply(
        logits.contiguous(), None if bias is None else bias.float().contiguous(), k, float(aux_coeff),
        float(z_coeff), load)
    return choice, w, aux, dict(row_of=row_of, src_of=src_of, grp_m=grp_m, grp_k=grp_k, P=src_of.numel(),
                                counts=counts)


def grouped_experts(x, choice, w, w_fc, w_proj, pl=None):
    """Routed-expert output sum_s w[t, s] expert_{choice[t, s]}(x[t]) for x [T, d] (CUDA).

    w_fc [E, F, d] and w_proj [E, d, F] are the stacked expert weights (any float dtype; the
    GEMMs run in bf16 with fp32 accumulation, gradients come back in the weights' dtype).  ``pl``:
    a row plan already made by ``fused_route``."""
    pl = pl or plan(choice, w_fc.shape[0])
    return _GroupedExperts.apply(x, w, w_fc, w_proj, pl["row_of"], pl["src_of"], pl["grp_m"], pl["grp_k"])


def grouped_experts_state(x, choice, w, moe, pl=None):
    """``grouped_experts`` on a layer's kernel state: the stacked bf16 shadows ``moe._w_fc`` /
    ``moe._w_proj`` are the operands and the weight gradients accumulate into the experts'
    ``main_grad`` stacks, so no per-forward stack or cast of the fp32 experts is made."""
    pl = pl or plan(choice, moe._w_fc.shape[0])
    return _GroupedExperts.apply(x, w, moe._w_fc, moe._w_proj, pl["row_of"], pl["src_of"], pl["grp_m"], pl["grp_k"],
                                 moe)
