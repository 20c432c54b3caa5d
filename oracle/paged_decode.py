"""fp32 CPU restatement of the paged-GQA decode -- TEST INFRASTRUCTURE ONLY.

paged_decode_ref restates the operator's mathematical definition (task.md:138-147) and
its token -> page mapping (task.md:94,146): for sequence b only the first
ceil(L_b / P) block-table entries are read, token t is slot t % P of page
block_table[b, t // P], and query head h reads KV head h // (Hq / Hkv).  Beyond the
reference's seqlen_q = 1 it also restates several query tokens per sequence with the
end-aligned causal mask of flash_attn_with_kvcache (the reference's comparison target,
task.md:16-26), which the run_kernel ABI can express through seqlen_q and causal.

split_partials_ref / lse_combine_ref restate the split-KV online softmax with a
running max (optimized_c500_flash_attn.cu:370-423: page max, alpha = exp(m_old - m_new),
weights, row sum) and the log-sum-exp merge of split partials
(optimized_c500_flash_attn.cu:681-727: global max over non-empty splits, then
sum l*beta and sum o*beta), in the log2 domain the CUDA kernel uses.

match_stats restates the reference's acceptance rule (verify_real.py:42-45,
task.md:151-156).
"""
import math

import numpy as np
import torch


def _gather_seq(k_cache, v_cache, block_table, b, L):
    P = k_cache.shape[1]
    n = (L + P - 1) // P
    pages = block_table[b, :n].to(torch.int64)
    Hkv, D = k_cache.shape[2], k_cache.shape[3]
    K = k_cache[pages].reshape(n * P, Hkv, D)[:L]
    V = v_cache[pages].reshape(n * P, Hkv, D)[:L]
    return K, V


def paged_decode_ref(q, k_cache, v_cache, block_table, seq_lens, scale=None, rows=None,
                     causal=False, return_lse=False):
    """fp32 reference.  q [B, Hq, D] (one query token) or [B, Sq, Hq, D]; pools
    [num_pages, P, Hkv, D].  Returns fp32 of q's shape.

    With Sq query tokens, token i of sequence b sees keys [0, L_b) -- or, when `causal`,
    keys [0, L_b - Sq + i] (the mask aligned to the end of the cache, as
    flash_attn_with_kvcache defines it).  A query with no visible key (L_b == 0, or
    causal with L_b - Sq + i < 0) gives zeros.  `rows` limits the work to the given
    sequence indices (the other rows stay zero).  With `return_lse` also returns
    lse [B, Hq, Sq] fp32: ln of the sum of exp(scale * q.k) over the visible keys (-inf
    for a query with none), as flash_attn_with_kvcache's softmax_lse."""
    squeeze = q.dim() == 3
    q4 = (q.unsqueeze(1) if squeeze else q).cpu()
    k_cache, v_cache = k_cache.cpu(), v_cache.cpu()
    block_table, seq_lens = block_table.cpu(), seq_lens.cpu()
    B, Sq, Hq, D = q4.shape
    Hkv = k_cache.shape[2]
    g = Hq // Hkv
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    out = torch.zeros(B, Sq, Hq, D, dtype=torch.float32)
    lse = torch.full((B, Hq, Sq), float("-inf"), dtype=torch.float32)
    for b in (range(B) if rows is None else rows):
        L = int(seq_lens[b])
        if L <= 0:
            continue
        K, V = _gather_seq(k_cache, v_cache, block_table, b, L)
        Kt = K.float().permute(1, 2, 0)            # [Hkv, D, L]
        Vt = V.float().permute(1, 0, 2)            # [Hkv, L, D]
        for i in range(Sq):
            n = L if not causal else min(L, L - Sq + i + 1)
            if n <= 0:
                continue
            qb = q4[b, i].float().reshape(Hkv, g, D)   # head h -> kv h // g
            s = torch.bmm(qb, Kt[:, :, :n]) * scale    # [Hkv, g, n]
            p = torch.softmax(s, dim=-1)
            out[b, i] = torch.bmm(p, Vt[:, :n]).reshape(Hq, D)
            lse[b, :, i] = torch.logsumexp(s, dim=-1).reshape(Hq)
    out = out[:, 0] if squeeze else out
    return (out, lse) if return_lse else out


def paged_decode_fp8_ref(q, k8, v8, k_scale, v_scale, block_table, seq_lens, scale=None,
                         causal=False, return_lse=False):
    """FP8 KV pages: the value of an element of KV head h is e4m3 * k_scale[h]
    (v_scale[h] for V).  The e4m3 bytes are decoded by torch's float8_e4m3fn conversion
    (OCP e4m3fn: bias 7, NaN = S.1111.111, no infinities), dequantised in fp32 and fed
    to paged_decode_ref."""
    Hkv = k8.shape[2]
    ks = torch.as_tensor(k_scale, dtype=torch.float32).reshape(-1).expand(Hkv).cpu()
    vs = torch.as_tensor(v_scale, dtype=torch.float32).reshape(-1).expand(Hkv).cpu()
    kd = k8.cpu().float() * ks.view(1, 1, Hkv, 1)
    vd = v8.cpu().float() * vs.view(1, 1, Hkv, 1)
    return paged_decode_ref(q, kd, vd, block_table, seq_lens, scale=scale, causal=causal,
                            return_lse=return_lse)


LOG2E = 1.4426950408889634


def split_partials_ref(q_row, K, V, scale, split_tokens, page_tokens=16, round_p_bf16=False):
    """Online-softmax partials of one (sequence, query head) row, numpy fp32.

    q_row [D]; K, V [L, D].  The sequence is cut into splits of `split_tokens`; each
    split walks `page_tokens`-token pages keeping a running max m (log2 domain), a
    rescaled row sum l and accumulator acc.  Returns lists (m, l, acc) per split."""
    q_row = np.asarray(q_row, dtype=np.float32)
    K = np.asarray(K, dtype=np.float32)
    V = np.asarray(V, dtype=np.float32)
    L = K.shape[0]
    c = np.float32(scale * LOG2E)
    parts = []
    for s0 in range(0, L, split_tokens):
        s1 = min(L, s0 + split_tokens)
        m = np.float32(-np.inf)
        l = np.float32(0.0)
        acc = np.zeros(K.shape[1], dtype=np.float32)
        for t0 in range(s0, s1, page_tokens):
            t1 = min(s1, t0 + page_tokens)
            s = (K[t0:t1] @ q_row) * c
            m_new = max(m, np.float32(s.max()))
            alpha = np.float32(np.exp2(m - m_new)) if np.isfinite(m) else np.float32(0.0)
            p = np.exp2(s - m_new).astype(np.float32)
            l = l * alpha + p.sum(dtype=np.float32)
            if round_p_bf16:
                p = torch.from_numpy(p).to(torch.bfloat16).float().numpy()
            acc = acc * alpha + p @ V[t0:t1]
            m = m_new
        parts.append((m, l, acc))
    return parts


def lse_combine_ref(parts):
    """Merge split partials: M = max m_s over splits with l_s > 0;
    out = sum_s 2^(m_s - M) acc_s / sum_s 2^(m_s - M) l_s."""
    live = [(m, l, a) for (m, l, a) in parts if l > 0]
    M = max(m for m, _, _ in live)
    den = sum(np.float32(np.exp2(m - M)) * l for m, l, _ in live)
    num = sum(np.float32(np.exp2(m - M)) * a for m, _, a in live)
    return (num / den).astype(np.float32)


def split_decode_ref(q, k_cache, v_cache, block_table, seq_lens, split_tokens, scale=None,
                     round_p_bf16=False):
    """Whole decode through split_partials_ref + lse_combine_ref (small cases only)."""
    q = q.reshape(q.shape[0], q.shape[-2], q.shape[-1]).cpu()
    B, Hq, D = q.shape
    Hkv = k_cache.shape[2]
    g = Hq // Hkv
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    out = np.zeros((B, Hq, D), dtype=np.float32)
    for b in range(B):
        L = int(seq_lens[b])
        if L <= 0:
            continue
        K, V = _gather_seq(k_cache.cpu(), v_cache.cpu(), block_table.cpu(), b, L)
        for h in range(Hq):
            kv = h // g
            parts = split_partials_ref(q[b, h].float().numpy(), K[:, kv].float().numpy(),
                                       V[:, kv].float().numpy(), scale, split_tokens,
                                       round_p_bf16=round_p_bf16)
            out[b, h] = lse_combine_ref(parts)
    return torch.from_numpy(out)


def match_stats(out, ref, atol=1.6e-2, rtol=1.6e-2):
    """The reference's acceptance statistics: fraction of elements with
    |out - ref| <= atol + rtol*|ref|, and whether any element exceeds 8x that bound."""
    out = out.float().cpu().reshape(-1)
    ref = ref.float().cpu().reshape(-1)
    tol = atol + rtol * ref.abs()
    diff = (out - ref).abs()
    ok = diff <= tol
    frac = ok.float().mean().item()
    outlier = bool((diff > 8 * tol).any().item()) or bool(torch.isnan(out).any().item())
    return frac, outlier, diff.max().item()
