"""Gated DeltaNet layer core (conv1d + delta rule + gated RMSNorm) with deferred MTP commit.

State of one request slot (all bf16):

* ``state [slots, Hv, dk, dv]`` - recurrent state after the committed tokens;
* ``conv_state [2, slots, conv_dim, 3]`` - last three raw conv inputs (ping-pong by
  the slot's ``parity``);
* ``pend_x [2, slots, P, conv_dim]`` / ``pend_ba [slots, P, 2*Hv]`` - raw inputs of
  the tokens of the last verify step that are not yet committed.

A step replays the first ``n_commit`` pending tokens, then processes its own tokens;
with ``keep_pending`` it stores the state *before* its own tokens and keeps their raw
inputs pending (speculative verify), otherwise it commits everything.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from ._ext import ext


def gdn_step(qkvz, ba, *, Hk, Hv, dk, dv, conv_w, A_log, dt_bias, norm_w, eps, state, conv_state, pend_x,
             pend_ba, parity, req_slot, q_start, n_commit, keep_pending, out, smem_state=False, status=None,
             host_meta=None):
    """Runs the GDN core for every request of the step; writes ``out [T, Hv*dv]`` (bf16).

    On the CPU path ``host_meta`` may carry the python lists
    ``(q_start, n_commit, keep_pending, req_slot, parity)`` to avoid tensor reads.
    """
    if qkvz.is_cuda:
        ext().gdn_step(qkvz, ba, Hk, Hv, dk, dv, conv_w, A_log, dt_bias, norm_w, float(eps), state, conv_state,
                       pend_x, pend_ba, parity, req_slot, q_start, n_commit, keep_pending, out, int(smem_state),
                       status)
        return out
    qs = q_start.tolist()
    nc = n_commit.tolist()
    kp = keep_pending.tolist()
    rs = req_slot.tolist()
    par = parity.tolist()
    r_ = Hv // Hk
    Kd = Hk * dk
    grp = 2 * dk + 2 * r_ * dv
    A = -torch.exp(A_log.float())
    for req in range(len(rs)):
        t0, T = qs[req], qs[req + 1] - qs[req]
        a = nc[req]
        if T + a <= 0:
            continue
        slot, p = rs[req], par[req]
        keep = bool(kp[req])
        # raw inputs of the tokens to run, in conv channel order [q heads | k heads | v heads]
        xs, bas, zs = [], [], []
        for i in range(a):
            xs.append(pend_x[p, slot, i].float())
            bas.append(pend_ba[slot, i].float())
            zs.append(None)
        for t in range(T):
            row = qkvz[t0 + t].float().view(Hk, grp)
            q = row[:, :dk].reshape(-1)
            k = row[:, dk:2 * dk].reshape(-1)
            v = row[:, 2 * dk:2 * dk + r_ * dv].reshape(-1)
            z = row[:, 2 * dk + r_ * dv:].reshape(Hv, dv)
            xs.append(torch.cat([q, k, v]))
            b_row = ba[t0 + t].float().view(Hk, 2 * r_)
            bas.append(torch.cat([b_row[:, :r_].reshape(-1), b_row[:, r_:].reshape(-1)]))
            zs.append(z)
        win = conv_state[p, slot].float().clone()  # [conv_dim, 3]
        S = state[slot].float().clone()  # [Hv, dk, dv]
        S_commit = None
        win_commit = win.clone() if (keep and a == 0) else None
        if keep:
            for t in range(T):
                pend_x[1 - p, slot, t] = xs[a + t].to(pend_x.dtype)
                pend_ba[slot, t] = bas[a + t].to(pend_ba.dtype)
        for idx, (x, bb, z) in enumerate(zip(xs, bas, zs)):
            full = torch.cat([win, x.unsqueeze(1)], 1)  # [conv_dim, 4]
            y = F.silu((full * conv_w.float()).sum(-1))
            win = full[:, 1:]
            q = y[:Kd].view(Hk, dk)
            k = y[Kd:2 * Kd].view(Hk, dk)
            v = y[2 * Kd:].view(Hv, dv)
            q = q * torch.rsqrt((q * q).sum(-1, keepdim=True) + 1e-6) / dk ** 0.5
            k = k * torch.rsqrt((k * k).sum(-1, keepdim=True) + 1e-6)
            q = q.repeat_interleave(r_, 0)
            k = k.repeat_interleave(r_, 0)
            beta = torch.sigmoid(bb[:Hv])
            g = torch.exp(A * F.softplus(bb[Hv:] + dt_bias.float()))
            S = S * g.view(Hv, 1, 1)
            kv = torch.einsum("hij,hi->hj", S, k)
            d = beta.unsqueeze(1) * (v - kv)
            S = S + k.unsqueeze(2) * d.unsqueeze(1)
            if idx >= a:
                o = torch.einsum("hij,hi->hj", S, q)
                o = o * torch.rsqrt(o.pow(2).mean(-1, keepdim=True) + eps)
                o = o.to(torch.bfloat16).float() * norm_w.float()
                o = o * F.silu(z)
                out[t0 + idx - a] = o.reshape(-1).to(out.dtype)
            if keep and idx == a - 1:
                S_commit = S.clone()
                win_commit = win.clone()
        if keep:
            if S_commit is not None:
                state[slot] = S_commit.to(state.dtype)
            conv_state[1 - p, slot] = win_commit.to(conv_state.dtype)
        else:
            state[slot] = S.to(state.dtype)
            conv_state[1 - p, slot] = win.to(conv_state.dtype)
    return out
