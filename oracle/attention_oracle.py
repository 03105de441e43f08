"""CPU oracle for the attention forward — TEST INFRASTRUCTURE ONLY.

This module is the checker, never the thing measured or shipped: only
``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import it.  The product path
(``flash_attention_sm75`` -> ``flash_attn_sm75_cuda`` -> ``libfa_b200.so``)
has no CPU fallback and never calls into this file.

It restates the reference's own CPU path, step for step:

* ``attention_reference`` follows src/reference/attention_ref.py:10-45 —
  fp32 upcast (:27-29), ``S = Q K^T * scale`` (:31), causal mask
  ``triu(ones, 1) -> -inf`` (:33-40), ``softmax`` (:42), ``P V`` (:43),
  ``.half()`` (:45).
* ``attention_fp32`` is the same algorithm kept in fp32 and extended with the
  row log-sum-exp ``LSE = logsumexp(S)`` (the reference has no LSE; this is
  the natural-log LSE of the same masked fp32 scores), the GQA head mapping of
  src/flash_attention_sm75/ops.py:6-27 (``repeat_interleave``: query head h
  reads KV head h // (Hq/Hkv)), an optional subset of query rows (for sizes
  whose full score matrix would not fit) and key-chunked evaluation.
* ``check`` restates src/reference/correctness.py:8-37 (max/mean abs and rel
  error, allclose) with the north-star tolerance.

Pinned against the reference: ``tests/golden/*.npz`` hold inputs and outputs
produced by importing the reference's ``attention_reference`` and
``_expand_kv_for_gqa`` (script: ``tests/golden/make_golden.py``);
``tests/test_oracle.py`` checks this module against every fixture.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import torch

# North-star tolerance for fp16/bf16 O against the fp32 oracle, applied
# elementwise as |err| <= ATOL + RTOL * |ref|; LSE absolute tolerance.
ATOL = 2e-3
RTOL = 1e-2
LSE_ATOL = 1e-4


def attention_reference(Q, K, V, causal=False, scale=None):
    """fp32 softmax(Q K^T * scale) V, returned as fp16 (attention_ref.py:10-45)."""
    if scale is None:
        scale = 1.0 / math.sqrt(Q.size(-1))
    Q_f = Q.float()
    K_f = K.float()
    V_f = V.float()
    S = torch.matmul(Q_f, K_f.transpose(-2, -1)) * scale
    if causal:
        seq_len = Q.size(-2)
        mask = torch.triu(torch.ones(seq_len, seq_len, device=Q.device, dtype=torch.bool),
                          diagonal=1)
        S.masked_fill_(mask, float("-inf"))
    P = torch.softmax(S, dim=-1)
    O = torch.matmul(P, V_f)
    return O.half()


def expand_kv_for_gqa(h_q: int, K: torch.Tensor, V: torch.Tensor):
    """K/V repeated to ``h_q`` heads in repeat_interleave order (ops.py:6-27)."""
    h_kv = K.size(1)
    if h_q == h_kv:
        return K, V
    if h_kv == 0 or h_q % h_kv != 0:
        raise RuntimeError(f"GQA expansion: Q heads ({h_q}) not divisible by K/V heads ({h_kv})")
    f = h_q // h_kv
    return K.repeat_interleave(f, dim=1), V.repeat_interleave(f, dim=1)


def attention_fp32(Q, K, V, causal=False, scale=None, rows: Optional[torch.Tensor] = None,
                   key_chunk: int = 4096, causal_offset: int = 0):
    """fp32 attention and LSE on the CPU.

    Q [B, Hq, Nq, d]; K, V [B, Hkv, Nk, d] (GQA by head mapping; Nk = Nq for
    the reference's square case).  Causal: key j is visible to query i iff
    j <= i + causal_offset (0 = the reference's top-left mask,
    attention_ref.py:33-40; Nk - Nq = bottom-right, the KV-cache convention).
    Rows that see no key get O = 0 and LSE = -inf.  ``rows`` is an optional
    1-D LongTensor of query indices evaluated (all if None).
    Returns (O fp32 [B, Hq, R, d], LSE fp32 [B, Hq, R]).
    """
    B, Hq, N, d = Q.shape
    Nk = K.size(2)
    if scale is None:
        scale = 1.0 / math.sqrt(d)
    K, V = expand_kv_for_gqa(Hq, K, V)
    q_idx = torch.arange(N) if rows is None else rows.to(torch.long)
    Qf = Q[:, :, q_idx, :].float()
    R = Qf.size(2)
    # online (chunked) softmax over keys, exact in fp32 up to summation order
    m = torch.full((B, Hq, R), float("-inf"))
    l = torch.zeros((B, Hq, R))
    acc = torch.zeros((B, Hq, R, d))
    for k0 in range(0, Nk, key_chunk):
        k1 = min(Nk, k0 + key_chunk)
        S = torch.matmul(Qf, K[:, :, k0:k1, :].float().transpose(-2, -1)) * scale
        if causal:
            key = torch.arange(k0, k1)
            S.masked_fill_(key[None, :] > q_idx[:, None] + causal_offset, float("-inf"))
        m_new = torch.maximum(m, S.amax(dim=-1))
        m_safe = torch.where(torch.isinf(m_new), torch.zeros_like(m_new), m_new)
        alpha = torch.exp(m - m_safe)
        P = torch.exp(S - m_safe[..., None])
        l = l * alpha + P.sum(dim=-1)
        acc = acc * alpha[..., None] + torch.matmul(P, V[:, :, k0:k1, :].float())
        m = m_new
    O = torch.where(l[..., None] > 0, acc / l.clamp_min(1e-38)[..., None], torch.zeros_like(acc))
    lse = torch.where(l > 0, m + torch.log(l), torch.full_like(l, float("-inf")))
    return O, lse


def kvcache_offset(Nq: int, Nk: int, mode: int) -> int:
    """Causal offset of fa_fwd_kvcache's FA_CAUSAL_* modes (1 bottom-right,
    2 top-left; 0 = not causal)."""
    return Nk - Nq if mode == 1 else 0


def attention_varlen_fp32(q, k, v, cu_q, cu_k, causal_mode: int = 0, scale=None):
    """fp32 attention of a packed variable-length batch, one sequence at a time.

    q [total_q, Hq, d], k/v [total_k, Hkv, d]; sequence b owns query rows
    [cu_q[b], cu_q[b+1]) and key rows [cu_k[b], cu_k[b+1]).  causal_mode:
    0 none, 1 bottom-right (j <= i + nk - nq), 2 top-left (j <= i), per
    sequence.  Returns (O fp32 [total_q, Hq, d], LSE fp32 [Hq, total_q]); rows
    outside every sequence stay O = 0, LSE = -inf.
    """
    Tq, Hq, d = q.shape
    O = torch.zeros((Tq, Hq, d))
    lse = torch.full((Hq, Tq), float("-inf"))
    cu_q = [int(x) for x in cu_q]
    cu_k = [int(x) for x in cu_k]
    for b in range(len(cu_q) - 1):
        q0, q1, k0, k1 = cu_q[b], cu_q[b + 1], cu_k[b], cu_k[b + 1]
        if q1 <= q0:
            continue
        Qs = q[q0:q1].permute(1, 0, 2)[None]
        Ks = k[k0:k1].permute(1, 0, 2)[None]
        Vs = v[k0:k1].permute(1, 0, 2)[None]
        o, l = attention_fp32(Qs, Ks, Vs, causal=causal_mode != 0, scale=scale,
                              causal_offset=kvcache_offset(q1 - q0, k1 - k0, causal_mode))
        O[q0:q1] = o[0].permute(1, 0, 2)
        lse[:, q0:q1] = l[0]
    return O, lse


def attention_padded_fp32(Q, K, V, q_start, q_end, k_start, k_end, causal_mode: int = 0,
                          scale=None):
    """fp32 attention of a padded batch: batch entry b attends from query rows
    [q_start[b], q_end[b]) to key rows [k_start[b], k_end[b]) of Q [B, Hq, Nq, d]
    and K/V [B, Hkv, Nk, d], with the causal rule of the full padded rows
    (1 bottom-right: j <= i + Nk - Nq; 2 top-left: j <= i).  Rows outside a
    query range stay O = 0, LSE = -inf.  Returns (O fp32 [B, Hq, Nq, d], LSE
    fp32 [B, Hq, Nq]).
    """
    B, Hq, Nq, d = Q.shape
    Nk = K.size(2)
    O = torch.zeros((B, Hq, Nq, d))
    lse = torch.full((B, Hq, Nq), float("-inf"))
    base = kvcache_offset(Nq, Nk, causal_mode)
    for b in range(B):
        q0, q1 = int(q_start[b]), int(q_end[b])
        k0, k1 = int(k_start[b]), int(k_end[b])
        if q1 <= q0:
            continue
        o, l = attention_fp32(Q[b:b + 1, :, q0:q1], K[b:b + 1, :, k0:k1], V[b:b + 1, :, k0:k1],
                              causal=causal_mode != 0, scale=scale,
                              causal_offset=base + q0 - k0)
        O[b, :, q0:q1] = o[0]
        lse[b, :, q0:q1] = l[0]
    return O, lse


# ------------------------------------------------------------------ inputs
@dataclass(frozen=True)
class AttnConfig:
    name: str
    B: int
    Hq: int
    Hkv: int
    N: int
    d: int
    causal: bool
    input_scale: float = 1.0
    k_outlier_frac: float = 0.0   # fraction of K rows per (b, h) scaled by k_outlier_scale
    k_outlier_scale: float = 8.0

    @property
    def flops(self) -> float:
        """Algorithmic FLOPs 4*B*H*N^2*d, halved for causal (reference convention,
        flash-attention-sm75-fused/src/flash_mha_v2.cu:573-574)."""
        f = 4.0 * self.B * self.Hq * self.N * self.N * self.d
        return f * 0.5 if self.causal else f

    @property
    def min_bytes(self) -> int:
        """Q + K + V + O at 2 bytes plus LSE at 4 bytes."""
        q = self.B * self.Hq * self.N * self.d * 2
        kv = 2 * self.B * self.Hkv * self.N * self.d * 2
        return 2 * q + kv + self.B * self.Hq * self.N * 4


# The five BASELINE.json configurations (C1..C5; C5 in full and causal form).
CONFIGS = {
    "c1": AttnConfig("c1", 1, 1, 1, 512, 64, False),
    "c2": AttnConfig("c2", 4, 12, 12, 1024, 64, False),
    "c3": AttnConfig("c3", 4, 8, 8, 2048, 64, True, input_scale=0.5),
    "c4": AttnConfig("c4", 2, 32, 8, 4096, 128, True),
    "c5": AttnConfig("c5", 4, 32, 32, 8192, 128, False, k_outlier_frac=0.01),
    "c5c": AttnConfig("c5c", 4, 32, 32, 8192, 128, True, k_outlier_frac=0.01),
}


def make_inputs(cfg: AttnConfig, seed: int = 42, dtype=torch.float16):
    """Seeded CPU inputs: Q, K, V drawn in that order from N(0,1) (as
    tests/test_flash_d128.py:16-19), times ``input_scale``; then, per (b, h),
    ``randperm(N)[:N*frac]`` K rows scaled by ``k_outlier_scale``."""
    g = torch.Generator().manual_seed(seed)
    Q = torch.randn(cfg.B, cfg.Hq, cfg.N, cfg.d, generator=g, dtype=torch.float32)
    K = torch.randn(cfg.B, cfg.Hkv, cfg.N, cfg.d, generator=g, dtype=torch.float32)
    V = torch.randn(cfg.B, cfg.Hkv, cfg.N, cfg.d, generator=g, dtype=torch.float32)
    if cfg.input_scale != 1.0:
        Q *= cfg.input_scale
        K *= cfg.input_scale
        V *= cfg.input_scale
    n_out = int(cfg.N * cfg.k_outlier_frac)
    if n_out > 0:
        for b in range(cfg.B):
            for h in range(cfg.Hkv):
                idx = torch.randperm(cfg.N, generator=g)[:n_out]
                K[b, h, idx, :] *= cfg.k_outlier_scale
    return Q.to(dtype), K.to(dtype), V.to(dtype)


def sample_rows(N: int, n: int, seed: int = 0, tile: int = 128) -> torch.Tensor:
    """Query rows for row-sampled checks: always 0, N-1 and the edges of every
    128-row tile boundary near the causal diagonal blocks, plus seeded random rows."""
    fixed = {0, N - 1}
    for t in range(0, N, tile):
        for r in (t - 1, t, t + 1, t + tile // 2):
            if 0 <= r < N:
                fixed.add(r)
    g = torch.Generator().manual_seed(seed)
    rnd = torch.randperm(N, generator=g)[: max(0, n)].tolist()
    return torch.tensor(sorted(fixed.union(rnd)), dtype=torch.long)


# ------------------------------------------------------------------ checks
def check(out: torch.Tensor, ref: torch.Tensor, atol: float = ATOL, rtol: float = RTOL):
    """Error metrics of ``out`` against fp32 ``ref`` (correctness.py:8-37) and the
    pass/fail of the elementwise bound |err| <= atol + rtol*|ref|."""
    o = out.float()
    r = ref.float()
    err = (o - r).abs()
    rel = err / (r.abs() + 1e-8)
    bound = atol + rtol * r.abs()
    return {
        "max_abs_err": err.max().item() if err.numel() else 0.0,
        "mean_abs_err": err.mean().item() if err.numel() else 0.0,
        "max_rel_err": rel.max().item() if rel.numel() else 0.0,
        "max_excess": (err - bound).max().item() if err.numel() else -1.0,
        "finite": bool(torch.isfinite(o).all().item()),
        "ok": bool(torch.isfinite(o).all().item() and (err <= bound).all().item()),
    }


def check_lse(lse: torch.Tensor, ref: torch.Tensor, atol: float = LSE_ATOL):
    err = (lse.float() - ref.float()).abs()
    m = err.max().item() if err.numel() else 0.0
    return {"max_abs_err": m, "ok": bool(m <= atol)}


def attention_grads_fp32(Q, K, V, dO, causal=False, scale=None):
    """dQ, dK, dV of the fp32 attention (attention_ref.py:10-45 restated with
    autograd) for the upstream gradient dO.  GQA K/V are expanded by
    repeat_interleave, so their gradients are summed over each group.
    Materialises the N x N scores: small sizes only."""
    B, Hq, N, d = Q.shape
    if scale is None:
        scale = 1.0 / math.sqrt(d)
    q = Q.detach().float().requires_grad_(True)
    k = K.detach().float().requires_grad_(True)
    v = V.detach().float().requires_grad_(True)
    kx, vx = expand_kv_for_gqa(Hq, k, v)
    s = torch.matmul(q, kx.transpose(-2, -1)) * scale
    if causal:
        mask = torch.triu(torch.ones(N, k.size(2), dtype=torch.bool), diagonal=1)
        s = s.masked_fill(mask, float("-inf"))
    o = torch.matmul(torch.softmax(s, dim=-1), vx)
    o.backward(dO.float())
    return q.grad, k.grad, v.grad


def attention_grads_formulas(Q, K, V, dO, causal=False, scale=None):
    """The same gradients from the FlashAttention-2 backward formulas
    (P, D = rowsum(dO * O), dS = P * (dP - D), dQ = scale dS K, dK = scale dS^T Q,
    dV = P^T dO), used to cross-check attention_grads_fp32."""
    B, Hq, N, d = Q.shape
    if scale is None:
        scale = 1.0 / math.sqrt(d)
    G = Hq // K.size(1)
    kx, vx = expand_kv_for_gqa(Hq, K.float(), V.float())
    q, do = Q.float(), dO.float()
    s = torch.matmul(q, kx.transpose(-2, -1)) * scale
    if causal:
        mask = torch.triu(torch.ones(N, K.size(2), dtype=torch.bool), diagonal=1)
        s = s.masked_fill(mask, float("-inf"))
    p = torch.softmax(s, dim=-1)
    o = torch.matmul(p, vx)
    dd = (do * o).sum(-1, keepdim=True)
    dv = torch.matmul(p.transpose(-2, -1), do)
    dp = torch.matmul(do, vx.transpose(-2, -1))
    ds = p * (dp - dd)
    dq = torch.matmul(ds, kx) * scale
    dk = torch.matmul(ds.transpose(-2, -1), q) * scale
    dk = dk.view(B, K.size(1), G, N, d).sum(2)
    dv = dv.view(B, K.size(1), G, N, d).sum(2)
    return dq, dk, dv
