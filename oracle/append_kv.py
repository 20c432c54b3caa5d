"""CPU restatement of the append-KV step -- TEST INFRASTRUCTURE ONLY.

flash_attn_with_kvcache(q, k_cache, v_cache, k, v, cache_seqlens, block_table, ...)
(the operator the reference is compared against, task.md:16-26, where k = v = None)
writes the new tokens k / v [B, S_new, Hkv, D] at positions
[cache_seqlens[b], cache_seqlens[b] + S_new) of sequence b before attending; token t of
sequence b lives in slot t % P of page block_table[b, t // P] (task.md:94,146).  The
reference's own path never appends, so this restatement has no golden vectors: it is
pure index arithmetic, checked bit for bit, and by the decode identity
decode(append(cache, new), L) == decode(cache', L + S_new) in the tests.
"""
import torch


def append_kv_ref(k_cache, v_cache, k_new, v_new, seq_lens, block_table):
    """Returns new (k_cache, v_cache) CPU tensors with the tokens written."""
    k = k_cache.cpu().clone()
    v = v_cache.cpu().clone()
    k_new, v_new = k_new.cpu(), v_new.cpu()
    bt, lens = block_table.cpu(), seq_lens.cpu()
    P = k.shape[1]
    B, S_new = k_new.shape[0], k_new.shape[1]
    for b in range(B):
        L0 = int(lens[b])
        for s in range(S_new):
            t = L0 + s
            pid = int(bt[b, t // P])
            k[pid, t % P] = k_new[b, s]
            v[pid, t % P] = v_new[b, s]
    return k, v
