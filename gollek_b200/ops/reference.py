"""Plain-PyTorch implementations of every hot op (CPU path and numerics oracle).

Each function has exactly the semantics of its sm_100a kernel in ``csrc/kernels``;
GPU tests compare the kernel against these run in fp32.

Paged KV-cache layout (one layer): ``[num_blocks, 2, num_kv_heads, block_size, head_dim]``
(index 0 = K, 1 = V). A token's slot is ``block_id * block_size + offset``. The
reference keeps ``[block][layer]`` slabs (core/optimization/gollek-plugin-kv-cache/…/
kvcache/PhysicalBlockPool.java:142-145); here each layer owns a contiguous pool so a
(block, head) pair is one contiguous ``block_size × head_dim`` tile that a kernel
reads with 16-byte vector loads.
"""
from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn.functional as F


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float, center: bool = False) -> torch.Tensor:
    xf = x.float()
    if center:  # bias-free LayerNorm
        xf = xf - xf.mean(-1, keepdim=True)
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()
    return y.to(x.dtype)


def fused_add_rms_norm(x: torch.Tensor, residual: torch.Tensor, w: torch.Tensor, eps: float,
                       center: bool = False):
    """residual += x (in place, in residual's dtype); returns rms_norm(residual) * w."""
    r = (x.float() + residual.float())
    residual.copy_(r.to(residual.dtype))
    return rms_norm(residual, w, eps, center)


def rope_kv_write(qkv: torch.Tensor, positions: torch.Tensor, cos_sin: torch.Tensor,
                  kv_cache: Optional[torch.Tensor], slot_mapping: torch.Tensor,
                  num_heads: int, num_kv_heads: int, head_dim: int, bias: Optional[torch.Tensor] = None,
                  q_norm: Optional[torch.Tensor] = None, k_norm: Optional[torch.Tensor] = None,
                  norm_eps: float = 1e-6) -> torch.Tensor:
    """Split fused QKV (+ bias), per-head RMSNorm of q/k when weights are given (QK-norm), apply
    NeoX RoPE to q and k, scatter k/v into the paged cache.

    qkv: [T, (H + 2*Hk) * D]; returns rotated q [T, H, D]. Slots < 0 are skipped (padding).
    """
    T = qkv.shape[0]
    H, Hk, D = num_heads, num_kv_heads, head_dim
    if bias is not None:
        qkv = (qkv.float() + bias.float()).to(qkv.dtype)
    q = qkv[:, : H * D].view(T, H, D)
    k = qkv[:, H * D: (H + Hk) * D].view(T, Hk, D)
    v = qkv[:, (H + Hk) * D:].view(T, Hk, D)
    if q_norm is not None:
        def hnorm(x, w):
            xf = x.float()
            return xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + norm_eps) * w.float()
        q, k = hnorm(q, q_norm), hnorm(k, k_norm)
    cs = cos_sin[positions.long()].float()
    R = cos_sin.shape[1]  # rotary dims (< D: the remaining dims pass through)
    cos, sin = cs[:, None, : R // 2], cs[:, None, R // 2:]

    def rot(x):
        xf = x.float()
        x1, x2 = xf[..., : R // 2], xf[..., R // 2: R]
        return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin, xf[..., R:]], -1)

    qr = rot(q).to(qkv.dtype)
    kr = rot(k).to(qkv.dtype)
    if kv_cache is not None:
        bs = kv_cache.shape[3]
        sm = slot_mapping.long()
        valid = sm >= 0
        blk, off = sm[valid] // bs, sm[valid] % bs
        kv_cache[blk, 0, :, off, :] = kr[valid].to(kv_cache.dtype)
        kv_cache[blk, 1, :, off, :] = v[valid].to(kv_cache.dtype)
    return qr


def paged_attention(q: torch.Tensor, kv_cache: torch.Tensor, block_tables: torch.Tensor,
                    seq_lens: torch.Tensor, query_start_loc: torch.Tensor, scale: float,
                    window: int = 0, softcap: float = 0.0) -> torch.Tensor:
    """Causal attention of each sequence's new queries over its paged KV.

    q: [T, H, D] (tokens of all sequences, concatenated); seq_lens[b] = total KV length
    of sequence b *including* its new tokens; query i of sequence b (q_len tokens) sits at
    absolute position ``seq_lens[b] - q_len + i`` and attends to KV positions ≤ that
    (and, with ``window`` > 0, > position - window). ``softcap`` > 0 maps the scaled scores
    through softcap · tanh(score / softcap) before the softmax.
    """
    T, H, D = q.shape
    Hk, bs = kv_cache.shape[2], kv_cache.shape[3]
    out = torch.empty(T, H, D, dtype=q.dtype, device=q.device)
    qsl = query_start_loc.tolist()
    lens = seq_lens.tolist()
    rep = H // Hk
    for b in range(len(lens)):
        s, e = qsl[b], qsl[b + 1]
        ql, L = e - s, lens[b]
        if ql == 0:
            continue
        nb = (L + bs - 1) // bs
        blocks = block_tables[b, :nb].long()
        k = kv_cache[blocks, 0].permute(0, 2, 1, 3).reshape(nb * bs, Hk, D)[:L].float()
        v = kv_cache[blocks, 1].permute(0, 2, 1, 3).reshape(nb * bs, Hk, D)[:L].float()
        k = k.repeat_interleave(rep, 1)
        v = v.repeat_interleave(rep, 1)
        qb = q[s:e].float()
        sc = torch.einsum("qhd,khd->hqk", qb, k) * scale
        if softcap > 0:
            sc = softcap * torch.tanh(sc / softcap)
        qpos = torch.arange(L - ql, L, device=q.device)
        kpos = torch.arange(L, device=q.device)
        masked = kpos[None, None, :] > qpos[None, :, None]
        if window > 0:
            masked = masked | (kpos[None, None, :] <= qpos[None, :, None] - window)
        sc = sc.masked_fill(masked, float("-inf"))
        out[s:e] = torch.einsum("hqk,khd->qhd", torch.softmax(sc, -1), v).to(q.dtype)
    return out


def gemm(a: torch.Tensor, b: torch.Tensor, residual: Optional[torch.Tensor] = None) -> torch.Tensor:
    """y = a @ b.T (+ residual); a [M, K], b [N, K] (nn.Linear layout)."""
    y = a.float() @ b.float().t()
    if residual is not None:
        y = y + residual.float()
    return y.to(a.dtype)


def interleave_gate_up(w_gate: torch.Tensor, w_up: torch.Tensor, group: int = 64) -> torch.Tensor:
    """Row-interleave gate/up weights in groups of ``group`` rows: [g0 u0 g1 u1 …].

    The SwiGLU GEMM epilogue then finds a gate row and its matching up row inside the
    same N-tile (tile n covers gate rows [n*group,(n+1)*group) and the same up rows).
    """
    F_, K = w_gate.shape
    assert F_ % group == 0
    g = w_gate.view(F_ // group, group, K)
    u = w_up.view(F_ // group, group, K)
    return torch.stack([g, u], 1).reshape(2 * F_, K)


def glu_act(g: torch.Tensor, act: str) -> torch.Tensor:
    """The gate activation of a gated FFN: ``silu`` (SwiGLU) or ``gelu_tanh`` (GeGLU)."""
    return F.silu(g) if act == "silu" else F.gelu(g, approximate="tanh")


def gemm_swiglu(a: torch.Tensor, w_gu: torch.Tensor, group: int = 64, act: str = "silu") -> torch.Tensor:
    """act(a @ Wg.T) * (a @ Wu.T) for gate/up weights interleaved by ``interleave_gate_up``."""
    y = a.float() @ w_gu.float().t()
    return glu_interleaved(y, group, act).to(a.dtype)


def glu_interleaved(y: torch.Tensor, group: int = 64, act: str = "silu") -> torch.Tensor:
    """act(gate) * up of a [M, 2F] product whose columns interleave gate/up in groups."""
    M = y.shape[0]
    y = y.float().view(M, -1, 2, group)
    return (glu_act(y[:, :, 0], act) * y[:, :, 1]).reshape(M, -1)


def silu_mul(x: torch.Tensor) -> torch.Tensor:
    d = x.shape[-1] // 2
    return (F.silu(x[..., :d].float()) * x[..., d:].float()).to(x.dtype)


def embedding(ids: torch.Tensor, table: torch.Tensor) -> torch.Tensor:
    return table[ids.long()]


def apply_penalties_triples(logits: torch.Tensor, triples: torch.Tensor, repetition: torch.Tensor,
                            frequency: torch.Tensor, presence: torch.Tensor) -> torch.Tensor:
    """In-place penalties from unique (row, token, count) triples, ``count`` = occurrences among
    the generated tokens: HF repetition penalty on every listed token (divide positive /
    multiply negative logits), then OpenAI frequency (``- f * count``) and presence (``- p`` when
    count > 0) penalties."""
    if triples.numel() == 0:
        return logits
    r, t, c = triples[:, 0].long(), triples[:, 1].long(), triples[:, 2].float()
    v = logits[r, t].float()
    rp = repetition[r].float()
    v = torch.where(v > 0, v / rp, v * rp)
    v = v - frequency[r].float() * c - presence[r].float() * (c > 0).float()
    logits[r, t] = v.to(logits.dtype)
    return logits


_M32 = 0xFFFFFFFF


def _mul32(x: torch.Tensor, c: int) -> torch.Tensor:
    """(x * c) mod 2^32 for int64 tensors holding uint32 values (no int64 overflow)."""
    lo = x * (c & 0xFFFF)
    hi = ((x * (c >> 16)) & 0xFFFF) << 16
    return (lo + hi) & _M32


def hash32(x: torch.Tensor) -> torch.Tensor:
    """32-bit xor-shift-multiply hash (same constants as the CUDA sampler)."""
    x = x & _M32
    x = x ^ (x >> 16)
    x = _mul32(x, 0x7FEB352D)
    x = x ^ (x >> 15)
    x = _mul32(x, 0x846CA68B)
    x = x ^ (x >> 16)
    return x


def sampling_uniforms(seed: int, offset: int, V: int, device="cpu") -> torch.Tensor:
    """The uniforms in (0, 1) the GPU sampler draws for token ids 0..V-1 at (seed, offset)."""
    s = torch.tensor([seed & _M32], dtype=torch.int64)
    o = torch.tensor([(offset + 0x9E3779B9) & _M32], dtype=torch.int64)
    mix = hash32(s ^ hash32(o))
    ids = torch.arange(V, dtype=torch.int64)
    h = hash32(mix ^ hash32(ids))
    return (((h >> 8).double() + 0.5) / 16777216.0).float().to(device)


def sample(logits: torch.Tensor, temperature: torch.Tensor, top_k: torch.Tensor, top_p: torch.Tensor,
           min_p: torch.Tensor, seeds: torch.Tensor, offsets: torch.Tensor) -> torch.Tensor:
    """Per-row sampling. temperature <= 0 → greedy argmax (lowest id on ties). Otherwise the
    survivors of top-k (k <= 0 = off), then min-p (p_i >= min_p * p_max), then top-p (the smallest
    highest-probability set whose renormalised mass reaches top_p) compete in an exponential race:
    argmax_i (x_i - max) / T + Gumbel(u_i), with u_i from ``sampling_uniforms(seed, offset)``.

    Same filter order as the reference sampler (runner/safetensor/gollek-safetensor-engine/…/
    generation/TokenSampler.java:62-208: temperature → top-k → top-p → draw); min-p follows the
    llama.cpp chain (runner/llamacpp/gollek-runner-llamacpp/…/LlamaHandles.java:174-203).
    """
    B, V = logits.shape
    out = torch.empty(B, dtype=torch.long, device=logits.device)
    lf = logits.float()
    for b in range(B):
        t = float(temperature[b])
        row = lf[b]
        m = float(row.max())
        if t <= 0.0:
            out[b] = int(torch.nonzero(row == m)[0])
            continue
        keep = torch.ones(V, dtype=torch.bool, device=row.device)
        k = int(top_k[b])
        if 0 < k < V:
            kth = row.topk(k).values[-1]
            keep &= row >= kth
        mp = float(min_p[b])
        if mp > 0:
            keep &= row >= m + t * math.log(mp)
        w = torch.exp((row - m) / t) * keep
        tp = float(top_p[b])
        if tp < 1.0:
            sw, si = w.sort(descending=True, stable=True)
            cum = sw.cumsum(0)
            target = tp * float(cum[-1])
            n_keep = int((cum < target).sum()) + 1
            thr = sw[min(n_keep, V) - 1]
            keep &= w >= thr
        u = sampling_uniforms(int(seeds[b]), int(offsets[b]), V, row.device)
        score = (row - m) / t - torch.log(-torch.log(u))
        score = torch.where(keep, score, torch.full_like(score, float("-inf")))
        out[b] = int(score.argmax())
    return out


def filtered_probs(logits: torch.Tensor, temperature: torch.Tensor, top_k: torch.Tensor, top_p: torch.Tensor,
                   min_p: torch.Tensor) -> torch.Tensor:
    """The distribution ``sample`` draws from, for every row at once (rows with temperature > 0):
    softmax((x - max) / T) restricted to the top-k, then min-p, then renormalised top-p survivors.
    Used by speculative decoding to accept or resample draft tokens exactly."""
    lf = logits.float()
    B, V = lf.shape
    t = temperature.float().clamp_min(1e-6)[:, None]
    m = lf.max(-1, keepdim=True).values
    keep = torch.ones_like(lf, dtype=torch.bool)
    k = top_k.long()
    kk = torch.where((k > 0) & (k < V), k, torch.full_like(k, V))
    kth = lf.sort(-1, descending=True).values.gather(1, (kk - 1)[:, None])
    keep &= lf >= kth
    mp = min_p.float()[:, None]
    keep &= torch.where(mp > 0, lf >= m + t * torch.log(mp.clamp_min(1e-30)), torch.ones_like(keep))
    w = torch.exp((lf - m) / t) * keep
    sw, _ = w.sort(dim=-1, descending=True, stable=True)
    cum = sw.cumsum(-1)
    target = top_p.float()[:, None] * cum[:, -1:]
    n_keep = (cum < target).sum(-1, keepdim=True) + 1
    thr = sw.gather(1, (n_keep.clamp_max(V) - 1))
    keep &= torch.where(top_p.float()[:, None] < 1.0, w >= thr, torch.ones_like(keep))
    w = w * keep
    return w / w.sum(-1, keepdim=True)


def attention_dense(q, k, v, causal=True, scale=None):
    """Dense GQA attention, q [S,H,D], k/v [S,Hk,D] (test helper)."""
    S, H, D = q.shape
    rep = H // k.shape[1]
    scale = scale or 1.0 / math.sqrt(D)
    k = k.repeat_interleave(rep, 1).float()
    v = v.repeat_interleave(rep, 1).float()
    s = torch.einsum("qhd,khd->hqk", q.float(), k) * scale
    if causal:
        s = s + torch.full((S, S), float("-inf"), device=q.device).triu(1)
    return torch.einsum("hqk,khd->qhd", torch.softmax(s, -1), v).to(q.dtype)


def gdn_gates(a: torch.Tensor, b: torch.Tensor, a_log: torch.Tensor, dt_bias: torch.Tensor):
    """alpha = exp(-exp(A_log) * softplus(a + dt_bias)), beta = sigmoid(b); a, b [T, Hg]."""
    alpha = torch.exp(-torch.exp(a_log.float()) * torch.nn.functional.softplus(a.float() + dt_bias.float()))
    return alpha, torch.sigmoid(b.float())


def gdn_scan(proj: torch.Tensor, state: torch.Tensor, slots: torch.Tensor, reset: torch.Tensor,
             query_start: torch.Tensor, a_log: torch.Tensor, dt_bias: torch.Tensor, Hg: int) -> torch.Tensor:
    """fp32 gated delta rule over varlen sequences (see csrc/kernels/gdn.cu); updates ``state`` in
    place and returns raw o [T, Hg, D]."""
    D = state.shape[-1]
    HD = Hg * D
    p = proj.float()
    T = p.shape[0]
    silu = torch.nn.functional.silu
    q = torch.nn.functional.normalize(silu(p[:, :HD].view(T, Hg, D)), dim=-1, eps=1e-6) / math.sqrt(D)
    k = torch.nn.functional.normalize(silu(p[:, HD:2 * HD].view(T, Hg, D)), dim=-1, eps=1e-6)
    v = silu(p[:, 2 * HD:3 * HD].view(T, Hg, D))
    alpha, beta = gdn_gates(p[:, 4 * HD:4 * HD + Hg], p[:, 4 * HD + Hg:4 * HD + 2 * Hg], a_log, dt_bias)
    out = torch.zeros(T, Hg, D, dtype=torch.float32, device=proj.device)
    qs = query_start.tolist()
    for i in range(len(qs) - 1):
        slot = int(slots[i])
        S = torch.zeros(Hg, D, D, device=proj.device) if int(reset[i]) else state[slot].float().clone()
        for t in range(qs[i], qs[i + 1]):
            S = alpha[t].view(Hg, 1, 1) * S
            u = beta[t].view(Hg, 1) * (v[t] - torch.einsum("hij,hi->hj", S, k[t]))
            S = S + k[t].unsqueeze(-1) * u.unsqueeze(1)
            out[t] = torch.einsum("hij,hi->hj", S, q[t])
        state[slot] = S.to(state.dtype)
    return out


def gdn_gated_norm(o: torch.Tensor, g: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """RMSNorm over each head of o [T, Hg, D] times w, times silu(g) [T, Hg*D]; returns [T, Hg*D]."""
    T, Hg, D = o.shape
    of = o.float()
    y = of * torch.rsqrt(of.pow(2).mean(-1, keepdim=True) + eps) * w.float()
    return (y.reshape(T, Hg * D) * torch.nn.functional.silu(g.float())).to(o.dtype)


def moe_route(logits: torch.Tensor, top_k: int, renorm: bool = True, scoring: str = "softmax",
              bias: Optional[torch.Tensor] = None, n_group: int = 1, topk_group: int = 1,
              scale: float = 1.0):
    """Router logits [T, E] (fp32) → (expert ids [T, k] int64, weights [T, k] fp32).

    ``softmax`` (Mixtral): top-k of the softmax, renormalised over the k. ``sigmoid`` (DeepSeek-V3):
    the choice score is sigmoid(logit) + bias; experts are split into ``n_group`` groups, each group
    scored by the sum of its two best choice scores, and the top-k is taken inside the ``topk_group``
    best groups (other experts' scores count as 0); the weights are the chosen experts' sigmoid
    scores (without the bias), renormalised when ``renorm``, times ``scale``. Ties go to the lower
    expert id (the CUDA router does the same)."""
    logits = logits.float()
    T, E = logits.shape
    if scoring == "softmax":
        probs = torch.softmax(logits, dim=-1)
        choice = probs
    else:
        probs = torch.sigmoid(logits)
        choice = probs + (bias.float() if bias is not None else 0.0)
    if n_group > 1:
        g = choice.view(T, n_group, E // n_group)
        gscore = g.topk(2, dim=-1).values.sum(-1)
        keep = _topk_lowest_index(gscore, topk_group)
        gmask = torch.zeros(T, n_group, dtype=torch.bool, device=logits.device)
        gmask.scatter_(1, keep, True)
        choice = choice.masked_fill(~gmask.repeat_interleave(E // n_group, dim=1), 0.0)
    ids = _topk_lowest_index(choice, top_k)
    w = probs.gather(1, ids)
    if renorm:
        w = w / (w.sum(-1, keepdim=True) + (1e-20 if scoring != "softmax" else 0.0))
    return ids, w * scale


def _topk_lowest_index(x: torch.Tensor, k: int) -> torch.Tensor:
    """Indices of the k largest entries per row, ties broken towards the lower index."""
    # stable sort on descending value keeps equal values in index order
    return torch.sort(x, dim=-1, descending=True, stable=True).indices[..., :k]
