"""TEST INFRASTRUCTURE ONLY: numpy restatement of one metalLLM training step
(config 5 model), the checker of metalllm_b200's training step.

Follows model.h:414-757 with the kernels of embed.metal, layernorm.metal,
attention.metal, mlp.metal, linear.metal, loss.metal and optimstep.metal, for
a batch of B sequences.  fp32 math; values are rounded to bf16 where the GPU
stores a bf16 buffer, so the comparison measures the kernels, not the
storage format.  PARITY UNPINNED (the reference runs only on Apple Metal).

Weights are a dict of float32 arrays keyed like the model's parameters
("embed", "pos", "layer0.qw", ..., "linw"), all already bf16-representable.
"""
from __future__ import annotations

import numpy as np

# Working precision of the restatement (float32 as the GPU; the oracle's own
# finite-difference self-test switches it to float64 with r16 disabled).
FLOAT = np.float32


def r16(x):
    """Round float32 values to the nearest bf16 (ties to even), as float32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32)
    # finite values stay below 2^32 after adding at most 0x8000
    r = (u >> np.uint32(16)) & np.uint32(1)
    r += np.uint32(0x7FFF)
    r += u
    r &= np.uint32(0xFFFF0000)
    return r.view(np.float32)


def layernorm(x, g, b, eps=1e-5):
    """layernorm.metal:10-71: returns (bf16 x_norm, bf16 out, fp32 stdev)."""
    mean = x.mean(axis=1, keepdims=True, dtype=np.float64).astype(FLOAT)
    var = ((x - mean) ** 2).mean(axis=1, keepdims=True, dtype=np.float64).astype(FLOAT)
    sd = np.sqrt(var + eps).astype(FLOAT)
    xn = (x - mean) / sd
    return r16(xn), r16(g * xn + b), sd[:, 0]


def layernorm_backward(dz, xn, g, sd):
    """layernorm.metal:74-127 (fp32): returns (bf16 dx, dgamma, dbeta)."""
    gg = dz * g
    m1 = gg.mean(axis=1, keepdims=True)
    m2 = (gg * xn).mean(axis=1, keepdims=True)
    dx = (gg - m1 - xn * m2) / sd[:, None]
    return r16(dx), (dz * xn).sum(axis=0), dz.sum(axis=0)


def attention(q, k, v, B, T, NH):
    """Causal attention per (batch, head): returns bf16 O [R, E] and lse [R, NH]."""
    E = q.shape[1]
    D = E // NH
    qh = q.reshape(B, T, NH, D).transpose(0, 2, 1, 3)
    kh = k.reshape(B, T, NH, D).transpose(0, 2, 1, 3)
    vh = v.reshape(B, T, NH, D).transpose(0, 2, 1, 3)
    s = (qh @ kh.transpose(0, 1, 3, 2)) / np.sqrt(D)
    mask = np.triu(np.ones((T, T), bool), 1)
    s = np.where(mask, -np.inf, s)
    m = s.max(-1, keepdims=True)
    p = np.exp(s - m)
    l = p.sum(-1, keepdims=True)
    o = (p / l) @ vh
    lse = (m + np.log(l))[..., 0]                       # [B, NH, T]
    return (r16(o.transpose(0, 2, 1, 3).reshape(B * T, E)),
            lse.transpose(0, 2, 1).reshape(B * T, NH).astype(FLOAT))


def attention_backward(dO, O, lse, q, k, v, B, T, NH):
    """computeD + flashAttentionBackward: (bf16 D, fp32 dQ, bf16 dK, bf16 dV)."""
    E = q.shape[1]
    D = E // NH
    sh = lambda a: a.reshape(B, T, NH, D).transpose(0, 2, 1, 3)
    qh, kh, vh, doh, oh = sh(q), sh(k), sh(v), sh(dO), sh(O)
    Dv = r16((doh * oh).sum(-1))                          # [B, NH, T]
    lh = lse.reshape(B, T, NH).transpose(0, 2, 1)
    s = (qh @ kh.transpose(0, 1, 3, 2)) / np.sqrt(D)
    mask = np.triu(np.ones((T, T), bool), 1)
    p = np.where(mask, 0.0, np.exp(s - lh[..., None]))
    dp = doh @ vh.transpose(0, 1, 3, 2)
    ds = p * (dp - Dv[..., None]) / np.sqrt(D)
    un = lambda a: a.transpose(0, 2, 1, 3).reshape(B * T, E).astype(FLOAT)
    return (Dv, un(ds @ kh), r16(un(ds.transpose(0, 1, 3, 2) @ qh)),
            r16(un(p.transpose(0, 1, 3, 2) @ doh)))


def forward_backward(W, tok, tgt, B, T, NH, L, masks=None):
    """One forward + backward: returns (mean loss, logits, grads dict).

    masks (optional, one bool [B*T, hidden] per layer) replaces the ReLU masks
    of the MLPs: activations that round to opposite signs near zero on the
    checked implementation would otherwise flip whole gradient entries."""
    R = B * T
    f32 = FLOAT
    h = r16(W["embed"][tok.reshape(-1)] + W["pos"][np.arange(R) % T])
    cache = []
    for n in range(L):
        P = lambda k: W[f"layer{n}.{k}"]
        xn1, ln1, sd1 = layernorm(h, P("ln1_gamma"), P("ln1_beta"))
        q, k, v = r16(ln1 @ P("qw")), r16(ln1 @ P("kw")), r16(ln1 @ P("vw"))
        att, lse = attention(q, k, v, B, T, NH)
        po = r16(att @ P("projw"))
        res1 = r16(h + po)
        xn2, ln2, sd2 = layernorm(res1, P("ln2_gamma"), P("ln2_beta"))
        mv = r16(ln2 @ P("up"))
        mask = mv > 0 if masks is None else np.asarray(masks[n], bool)
        mv = np.where(mask, mv, 0).astype(f32)
        mo = r16(mv @ P("dp"))
        res2 = r16(res1 + mo)
        cache.append((h, xn1, ln1, sd1, q, k, v, att, lse, res1, xn2, ln2, sd2, mv, mask))
        h = res2
    xnf, lnf, sdf = layernorm(h, W["lnf_gamma"], W["lnf_beta"])
    logits = r16(lnf @ W["linw"])
    mx = logits.max(1, keepdims=True)
    lse_r = (mx + np.log(np.exp(logits - mx).sum(1, keepdims=True)))[:, 0]
    y = tgt.reshape(-1)
    loss = float((lse_r - logits[np.arange(R), y]).mean())
    # backward (model.h:537-711)
    G = {}
    prob = np.exp(logits - lse_r[:, None])
    onehot = np.zeros_like(prob)
    onehot[np.arange(R), y] = 1
    dlog = r16((prob - onehot) / R)
    ds = r16(dlog @ W["linw"].T)
    G["linw"] = r16(lnf.T @ dlog)
    ds, G["lnf_gamma"], G["lnf_beta"] = layernorm_backward(ds, xnf, W["lnf_gamma"], sdf)
    for n in reversed(range(L)):
        P = lambda k: W[f"layer{n}.{k}"]
        (hin, xn1, ln1, sd1, q, k, v, att, lse, res1, xn2, ln2, sd2, mv, mask) = cache[n]
        dmv = np.where(mask, r16(ds @ P("dp").T), 0).astype(f32)
        G[f"layer{n}.up"] = r16(ln2.T @ dmv)
        G[f"layer{n}.dp"] = r16(mv.T @ ds)
        db = r16(dmv @ P("up").T)
        db, G[f"layer{n}.ln2_gamma"], G[f"layer{n}.ln2_beta"] = layernorm_backward(db, xn2, P("ln2_gamma"), sd2)
        db = r16(db + ds)
        G[f"layer{n}.projw"] = r16(att.T @ db)
        dz = r16(db @ P("projw").T)
        _, dq, dk, dv = attention_backward(dz, att, lse, q, k, v, B, T, NH)
        dx = dq @ P("qw").T + dk @ P("kw").T + dv @ P("vw").T
        G[f"layer{n}.qw"] = ln1.T @ dq
        G[f"layer{n}.kw"] = r16(ln1.T @ dk)
        G[f"layer{n}.vw"] = r16(ln1.T @ dv)
        ds = r16(dx)
        ds, G[f"layer{n}.ln1_gamma"], G[f"layer{n}.ln1_beta"] = layernorm_backward(ds, xn1, P("ln1_gamma"), sd1)
        ds = r16(ds + db)
    demb = np.zeros_like(W["embed"])
    np.add.at(demb, tok.reshape(-1), ds)
    G["embed"] = demb
    G["pos"] = r16(ds.reshape(B, T, -1).sum(0))
    return loss, logits, G


def adam(master, grad_bf16, m, v, step, lr):
    """optimstep.metal:15-42 on flat arrays (bf16 moments), returns new (p, m, v)."""
    b1, b2, eps = np.float32(0.9), np.float32(0.999), np.float32(1e-8)
    lr_t = np.float32(lr * np.sqrt(1.0 - 0.999 ** step) / (1.0 - 0.9 ** step))
    g = grad_bf16.astype(np.float32)
    vi = b2 * v + np.float32(0.001) * (g * g)
    mi = b1 * m + np.float32(0.1) * g
    p = master - lr_t * mi / np.sqrt(vi + eps)
    return p.astype(np.float32), r16(mi), r16(vi)
