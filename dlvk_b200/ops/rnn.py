"""Recurrent layers' compute: one autograd node per (bi)directional layer.

Forward, per direction (weights W_ih [G*H, I], W_hh [G*H, H], biases [G*H];
gate order LSTM i,f,g,o and GRU r,z,n as in
include/dlvk/layers/recurrent_layers.h:18-200):

  xproj = x W_ih^T + b            one tensor-core GEMM over all B*T rows
  for t in order:                 (reverse order for the backward direction)
      a_t = h_{t-1} W_hh^T + xproj_t      GEMM, the add fused in its epilogue
      h_t = cell(a_t)                     rnn.cu element-wise kernel

Backward (BPTT):

  for t in reversed(order):
      dA_t = cell_bwd(dh_t, saved_t)
      dh_{t-1} = dA_t W_hh + dY_{t-1}     GEMM, dY added in the epilogue
  dW_ih = dA^T X,  dW_hh = dA^T H_prev,  dX = dA W_ih    three GEMMs over all steps
  db = column sums of dA

Both directions of a bidirectional layer write their half of the [B, T, 2H]
output in place (strided row views), so there is no concat and no flip.
The CPU path runs the same loop with the cell math in torch (the oracle).
"""
from __future__ import annotations

from typing import List, Optional

import torch

from . import core as K

KINDS = {"rnn": 0, "lstm": 1, "gru": 2}
GATES = {0: 1, 1: 4, 2: 3}


def _rnn():
    return K.N().rnn


# ---------------------------------------------------------------- CPU cell math (oracle)
def _cell_fwd_cpu(kind, H, a, hg, h_prev, c_prev, h_out, h_copy, c_out, saved):
    af = a.float()
    if kind == 0:
        h = torch.tanh(af)
    elif kind == 1:
        i, f = torch.sigmoid(af[:, :H]), torch.sigmoid(af[:, H:2 * H])
        g, o = torch.tanh(af[:, 2 * H:3 * H]), torch.sigmoid(af[:, 3 * H:])
        cp = c_prev.float() if c_prev is not None else torch.zeros_like(i)
        c = f * cp + i * g
        h = o * torch.tanh(c)
        c_out.copy_(c)
        saved.copy_(torch.cat([i, f, g, o], 1))
    else:
        hf = hg.float()
        r = torch.sigmoid(af[:, :H] + hf[:, :H])
        z = torch.sigmoid(af[:, H:2 * H] + hf[:, H:2 * H])
        hn = hf[:, 2 * H:]
        n = torch.tanh(af[:, 2 * H:] + r * hn)
        hp = h_prev.float() if h_prev is not None else torch.zeros_like(n)
        h = (1 - z) * n + z * hp
        saved.copy_(torch.cat([r, z, n, hn], 1))
    h_out.copy_(h)
    if h_copy is not None:
        h_copy.copy_(h)


def _cell_bwd_cpu(kind, H, dh, dc_next, h_t, h_prev, c_t, c_prev, saved, dA, dAh, dc_prev, dy_prev, resid):
    g = dh.float()
    if kind == 0:
        h = h_t.float()
        dA.copy_(g * (1 - h * h))
        return
    sv = saved
    if kind == 1:
        i, f, gg, o = sv[:, :H], sv[:, H:2 * H], sv[:, 2 * H:3 * H], sv[:, 3 * H:]
        tc = torch.tanh(c_t)
        dc = g * o * (1 - tc * tc)
        if dc_next is not None:
            dc = dc + dc_next
        cp = c_prev if c_prev is not None else torch.zeros_like(dc)
        dA.copy_(torch.cat([dc * gg * i * (1 - i), dc * cp * f * (1 - f), dc * i * (1 - gg * gg),
                            g * tc * o * (1 - o)], 1))
        dc_prev.copy_(dc * f)
        return
    r, z, n, hn = sv[:, :H], sv[:, H:2 * H], sv[:, 2 * H:3 * H], sv[:, 3 * H:]
    hp = h_prev.float() if h_prev is not None else torch.zeros_like(n)
    dn = g * (1 - z) * (1 - n * n)
    dz = g * (hp - n) * z * (1 - z)
    dr = dn * hn * r * (1 - r)
    dA.copy_(torch.cat([dr, dz, dn], 1))
    dAh.copy_(torch.cat([dr, dz, dn * r], 1))
    if resid is not None:
        rv = g * z
        if dy_prev is not None:
            rv = rv + dy_prev.float()
        resid.copy_(rv)


def _cell_fwd(cuda, *args):
    if cuda:
        _rnn().cell_fwd(*args)
    else:
        _cell_fwd_cpu(*args)


def _cell_bwd(cuda, *args):
    if cuda:
        _rnn().cell_bwd(*args)
    else:
        _cell_bwd_cpu(*args)


# ---------------------------------------------------------------- one direction
class _Dir:
    """Parameters and saved activations of one direction."""

    def __init__(self, cell, reverse: bool):
        self.cell = cell          # the layer owning w_ih, w_hh, b_ih, b_hh
        self.reverse = reverse


def _order(T, reverse):
    return list(range(T - 1, -1, -1)) if reverse else list(range(T))


def _forward_dir(d: _Dir, x2, B, T, Y, h0, c0):
    cell = d.cell
    kind, H = cell.kind, cell.hidden_size
    G = GATES[kind]
    dt = x2.dtype
    dev = x2.device
    cuda = x2.is_cuda
    w_ih, w_hh, b_ih, b_hh = cell.w_ih, cell.w_hh, cell.b_ih, cell.b_hh
    if kind == 2:
        bias = b_ih.master if b_ih is not None else None
    elif b_ih is not None:
        bias = K.binary(b_ih.master.contiguous(), b_hh.master.contiguous(), K.BIN_ADD)
    else:
        bias = None
    xproj = K.gemm(x2, w_ih.value.t(), bias=bias).view(B, T, G * H)
    Hp = torch.empty(B, T, H, dtype=dt, device=dev)
    order = _order(T, d.reverse)
    if h0 is None:
        Hp[:, order[0]].zero_()
    else:
        Hp[:, order[0]].copy_(h0)
    saved = torch.empty(B, T, 4 * H, dtype=torch.float32, device=dev) if kind else None
    C = torch.empty(B, T, H, dtype=torch.float32, device=dev) if kind == 1 else None
    buf = torch.empty(B, G * H, dtype=dt, device=dev)
    c_prev = c0
    for k, t in enumerate(order):
        hp = Hp[:, t]
        nxt = Hp[:, order[k + 1]] if k + 1 < T else None
        if kind in (0, 1):
            K.gemm(hp, w_hh.value.t(), residual=xproj[:, t], out=buf)
            _cell_fwd(cuda, kind, H, buf, None, None, c_prev, Y[:, t], nxt,
                      C[:, t] if C is not None else None, saved[:, t] if saved is not None else None)
            if C is not None:
                c_prev = C[:, t]
        else:
            K.gemm(hp, w_hh.value.t(), bias=b_hh.master if b_hh is not None else None, out=buf)
            _cell_fwd(cuda, kind, H, xproj[:, t], buf, hp, None, Y[:, t], nxt, None, saved[:, t])
    d.saved = (Hp, saved, C, c0)
    d.last_h = Y[:, order[-1]]
    d.last_c = C[:, order[-1]] if C is not None else None


def _param_grad(p, fn):
    """Run fn(out, beta) into p.grad honouring the accumulate flag."""
    acc = p.take_accumulate_flag()
    fn(p.grad, 1.0 if acc else 0.0, acc)
    p.grad_ready()


def _backward_dir(d: _Dir, x2, B, T, Y, dY, dX):
    cell = d.cell
    kind, H = cell.kind, cell.hidden_size
    G = GATES[kind]
    Hp, saved, C, c0 = d.saved
    dt = x2.dtype
    dev = x2.device
    cuda = x2.is_cuda
    dA = torch.empty(B, T, G * H, dtype=dt, device=dev)
    dAh = torch.empty(B, T, G * H, dtype=dt, device=dev) if kind == 2 else dA
    dh_buf = torch.empty(B, H, dtype=dt, device=dev)
    resid = torch.empty(B, H, dtype=dt, device=dev) if kind == 2 else None
    dcb = [torch.empty(B, H, dtype=torch.float32, device=dev) for _ in range(2)] if kind == 1 else None
    rev = list(reversed(_order(T, d.reverse)))
    for k, t in enumerate(rev):
        dh = dY[:, t] if k == 0 else dh_buf
        tp = rev[k + 1] if k + 1 < T else None
        c_prev = (C[:, tp] if tp is not None else c0) if kind == 1 else None
        _cell_bwd(cuda, kind, H, dh, dcb[(k - 1) % 2] if (kind == 1 and k > 0) else None,
                  Y[:, t] if kind == 0 else None, Hp[:, t] if kind == 2 else None,
                  C[:, t] if kind == 1 else None, c_prev, saved[:, t] if saved is not None else None,
                  dA[:, t], dAh[:, t] if kind == 2 else None, dcb[k % 2] if kind == 1 else None,
                  dY[:, tp] if (kind == 2 and tp is not None) else None,
                  resid if (kind == 2 and tp is not None) else None)
        if tp is not None:
            if kind == 2:
                K.gemm(dAh[:, t], cell.w_hh.value, residual=resid, out=dh_buf)
            else:
                K.gemm(dA[:, t], cell.w_hh.value, residual=dY[:, tp], out=dh_buf)
    dA2 = dA.view(B * T, G * H)
    dAh2 = dAh.view(B * T, G * H)
    _param_grad(cell.w_ih, lambda out, beta, acc: K.gemm(dA2.t(), x2, out=out, beta=beta, out_dtype=torch.float32))
    _param_grad(cell.w_hh, lambda out, beta, acc: K.gemm(dAh2.t(), Hp.view(B * T, H), out=out, beta=beta,
                                                         out_dtype=torch.float32))
    if cell.b_ih is not None:
        _param_grad(cell.b_ih, lambda out, beta, acc: K.colsum(dA2, out=out, accumulate=acc))
        _param_grad(cell.b_hh, lambda out, beta, acc: K.colsum(dAh2, out=out, accumulate=acc))
    if dX is None:
        return K.gemm(dA2, cell.w_ih.value)
    K.gemm(dA2, cell.w_ih.value, out=dX, beta=1.0)
    return dX


class RecurrentFn(torch.autograd.Function):
    """x [B, T, I] -> y [B, T, D*H] for D = len(cells) directions."""

    @staticmethod
    def forward(ctx, x, anchor, cells, reverse_flags, states):
        B, T, I = x.shape
        H = cells[0].hidden_size
        D = len(cells)
        x2 = x.contiguous().view(B * T, I)
        Y = torch.empty(B, T, D * H, dtype=x.dtype, device=x.device)
        dirs = []
        for di, (cell, rev) in enumerate(zip(cells, reverse_flags)):
            d = _Dir(cell, rev)
            h0, c0 = states[di] if states is not None else (None, None)
            _forward_dir(d, x2, B, T, Y[:, :, di * H:(di + 1) * H], h0, c0)
            dirs.append(d)
        ctx.dirs, ctx.x2, ctx.shape, ctx.Y = dirs, x2, (B, T, I, H), Y
        return Y

    @staticmethod
    def backward(ctx, gY):
        B, T, I, H = ctx.shape
        gY = gY.contiguous()
        dX = None
        for di, d in enumerate(ctx.dirs):
            dX = _backward_dir(d, ctx.x2, B, T, ctx.Y[:, :, di * H:(di + 1) * H], gY[:, :, di * H:(di + 1) * H], dX)
        ctx.dirs = None
        return dX.view(B, T, I), None, None, None, None
