"""Seeded synthetic inputs for the paged-GQA decode.

Two families:

* `baseline_config(name)` - the five workloads named by the benchmark
  (c1 ... c5: shapes, seq-len distributions, pool sizes and page permutations).
* `spj_case(n)` - the reference's 14-case correctness table (verify_real.py:8-10) with its
  seq-len rule (verify_real.py:21-26: torch.manual_seed(42); lengths randint[1, cap],
  lengths[0] = cap, lengths[1] = 1 when B > 1, case 1 all ones) and its contiguous
  block table (verify_real.py:30), optionally with a permuted table instead.

Inputs are generated on the CPU with torch's seeded generator (bit-reproducible for a
given torch build) or, for sizes the host cannot hold comfortably, directly on a CUDA
device.  There is no public dataset behind these workloads; the shapes and value
distributions are those the benchmark names.
"""
import dataclasses
import hashlib
import math
from typing import Optional

import torch

HEAD_DIM = 128


@dataclasses.dataclass
class DecodeInputs:
    q: torch.Tensor            # [B, Hq, D] bf16
    k: torch.Tensor            # [num_pages, P, Hkv, D] bf16
    v: torch.Tensor            # [num_pages, P, Hkv, D] bf16
    block_table: torch.Tensor  # [B, stride] int32
    seq_lens: torch.Tensor     # [B] int32
    scale: float
    name: str = ""
    seqlen_k: int = 0          # capacity the reference ABI passes as seqlen_k
    k_scale: Optional[torch.Tensor] = None  # FP8 pools: [Hkv] float32 dequantisation factors
    v_scale: Optional[torch.Tensor] = None

    @property
    def batch(self):
        return self.q.shape[0]

    @property
    def num_heads(self):
        return self.q.shape[-2]  # q is [B, Hq, D] or [B, Sq, Hq, D]

    @property
    def num_heads_k(self):
        return self.k.shape[2]

    @property
    def page_size(self):
        return self.k.shape[1]

    @property
    def num_pages(self):
        return self.k.shape[0]

    def kv_bytes(self):
        """Algorithmic K+V bytes of one call: sum_b L_b * Hkv * D * (element bytes) * 2."""
        return (int(self.seq_lens.to(torch.int64).sum().item()) * self.num_heads_k * HEAD_DIM
                * 2 * self.k.element_size())

    def algorithmic_bytes(self):
        """KV bytes + q and out + the block-table entries and lengths actually read."""
        q_elems = self.q.numel()  # [B, (Sq,) Hq, D]: q read and out written once each
        pages = int(((self.seq_lens.to(torch.int64) + self.page_size - 1)
                     // self.page_size).sum().item())
        return self.kv_bytes() + 2 * q_elems * 2 + pages * 4 + self.batch * 4

    def to(self, device):
        mv = (lambda t: None if t is None else t.to(device))
        return dataclasses.replace(
            self, q=self.q.to(device), k=self.k.to(device), v=self.v.to(device),
            block_table=self.block_table.to(device), seq_lens=self.seq_lens.to(device),
            k_scale=mv(self.k_scale), v_scale=mv(self.v_scale))

    def digest(self):
        """sha256 over every input byte (detects generator drift between machines)."""
        h = hashlib.sha256()
        for t in (self.q, self.k, self.v, self.block_table, self.seq_lens):
            h.update(t.detach().contiguous().cpu().view(torch.uint8).numpy().tobytes())
        return h.hexdigest()


def _randn(shape, gen, device, std=1.0):
    x = torch.randn(shape, generator=gen, device=device, dtype=torch.float32)
    if std != 1.0:
        x.mul_(std)
    return x.to(torch.bfloat16)


def _randn_bf16_large(shape, gen, device, std=1.0):
    """bf16 normal samples without an fp32 copy of the whole tensor (for GPU pools)."""
    out = torch.empty(shape, dtype=torch.bfloat16, device=device)
    flat = out.view(-1)
    step = 1 << 28
    for s in range(0, flat.numel(), step):
        e = min(flat.numel(), s + step)
        chunk = torch.randn(e - s, generator=gen, device=device, dtype=torch.float32)
        if std != 1.0:
            chunk.mul_(std)
        flat[s:e].copy_(chunk)
    return out


def _generator(seed, device):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def build_table(seq_lens, page_size, width, num_pages, gen, mode="permuted", pad="random"):
    """Block table [B, width] for the given lengths.

    mode "contiguous": sequence b owns pages [b*width, b*width + width) (the reference's
                       arange table, verify_real.py:30).
    mode "permuted":   the valid pages of all sequences are a random permutation of the
                       pool (num_pages >= total valid pages; the rest stay unused).
    pad:  padding slots get "random" valid page ids (they must never be read) or
          "zero" (page 0).
    """
    B = seq_lens.shape[0]
    npg = [(int(L) + page_size - 1) // page_size for L in seq_lens.tolist()]
    bt = torch.zeros(B, width, dtype=torch.int32)
    if mode == "contiguous":
        bt = torch.arange(B * width, dtype=torch.int32).reshape(B, width)
        return bt
    total = sum(npg)
    if total > num_pages:
        raise ValueError("pool too small for the lengths")
    perm = torch.randperm(num_pages, generator=gen).to(torch.int32)
    pos = 0
    for b in range(B):
        bt[b, :npg[b]] = perm[pos:pos + npg[b]]
        pos += npg[b]
        if width > npg[b]:
            if pad == "random":
                bt[b, npg[b]:] = torch.randint(0, num_pages, (width - npg[b],), generator=gen,
                                               dtype=torch.int32)
    return bt


# --------------------------------------------------------------------------------------
# The benchmark's five workloads
# --------------------------------------------------------------------------------------

CONFIGS = {
    "c1": dict(B=4, Hq=32, Hkv=8, P=16, desc="CPU-runnable case: L=1024 each, pool 256+16 pages"),
    "c2": dict(B=2, Hq=64, Hkv=8, P=16, desc="long context: L=32768 each, pool 4096+64 pages"),
    "c3": dict(B=256, Hq=32, Hkv=8, P=16, desc="large batch: L~U[128,2048], pool=sum ceil(L/16)"),
    "c4": dict(B=64, Hq=28, Hkv=4, P=64, desc="ragged g=7: L log-uniform [64,65536], 10% spare pages"),
    "c5": dict(B=512, Hq=64, Hkv=8, P=16, desc="8-GPU: L=16384 fixed, ~34 GB pool"),
}


def config_seq_lens(name, seed=0):
    cfg = CONFIGS[name]
    B = cfg["B"]
    g = _generator(seed + 1, "cpu")
    if name == "c1":
        return torch.full((B,), 1024, dtype=torch.int32), 1024
    if name == "c2":
        return torch.full((B,), 32768, dtype=torch.int32), 32768
    if name == "c3":
        return torch.randint(128, 2049, (B,), generator=g, dtype=torch.int32), 2048
    if name == "c4":
        u = torch.rand(B, generator=g, dtype=torch.float64)
        L = torch.exp(math.log(64) + u * (math.log(65536) - math.log(64)))
        L = L.round().clamp(64, 65536).to(torch.int32)
        return L, 65536
    if name == "c5":
        return torch.full((B,), 16384, dtype=torch.int32), 16384
    raise KeyError(name)


def baseline_config(name, seed=0, device="cpu", kv_head_range: Optional[tuple] = None,
                    batch_limit: Optional[int] = None):
    """Inputs of workload `name` (c1..c5).

    kv_head_range=(lo, hi) builds only KV heads [lo, hi) and their query heads (the
    shard a GPU owns when the op is split by KV head); the page permutation and lengths
    are those of the full workload.  batch_limit keeps only the first sequences (the
    bounded CPU-baseline sample) with the same per-sequence data layout.
    """
    cfg = CONFIGS[name]
    B, Hq, Hkv, P = cfg["B"], cfg["Hq"], cfg["Hkv"], cfg["P"]
    D = HEAD_DIM
    gq = Hq // Hkv
    seq_lens, cap = config_seq_lens(name, seed)
    width = (cap + P - 1) // P
    npg = (seq_lens.to(torch.int64) + P - 1) // P
    used = int(npg.sum().item())
    if name == "c1":
        num_pages = used + 16
    elif name == "c2":
        num_pages = used + 64
    elif name == "c4":
        num_pages = used + (used + 9) // 10
    else:
        num_pages = used
    if num_pages % B == 0 and num_pages // B >= width:
        width = num_pages // B  # the reference ABI's row width (num_blocks / batch_size)
    gtab = _generator(seed + 2, "cpu")
    bt = build_table(seq_lens, P, width, num_pages, gtab, mode="permuted")
    if batch_limit is not None and batch_limit < B:
        # keep the first sequences and compact their pages into a small pool
        seq_lens = seq_lens[:batch_limit].clone()
        bt_full = bt[:batch_limit]
        npg_b = npg[:batch_limit].tolist()
        ids = torch.cat([bt_full[b, :npg_b[b]] for b in range(batch_limit)]).to(torch.int64)
        remap = {int(p): i for i, p in enumerate(ids.tolist())}
        bt = torch.zeros(batch_limit, width, dtype=torch.int32)
        for b in range(batch_limit):
            for i in range(npg_b[b]):
                bt[b, i] = remap[int(bt_full[b, i])]
        num_pages = len(ids)
        B = batch_limit
    lo, hi = kv_head_range if kv_head_range is not None else (0, Hkv)
    hk = hi - lo
    std_kv = 0.5 if name == "c4" else 1.0
    gdev = _generator(seed + 3 + 1000 * lo, device)
    big = device != "cpu"
    mk = _randn_bf16_large if big else _randn
    q = mk((B, hk * gq, D), gdev, device)
    k = mk((num_pages, P, hk, D), gdev, device, std_kv)
    v = mk((num_pages, P, hk, D), gdev, device, std_kv)
    return DecodeInputs(q=q, k=k, v=v, block_table=bt.to(device), seq_lens=seq_lens.to(device),
                        scale=1.0 / math.sqrt(D), name=name, seqlen_k=cap)


def golden_slice(name, index, seed=5):
    """A reduced batch of workload `name`: the sequences at `index` (their lengths), with
    the workload's head layout, page size and value distribution, a randomly permuted
    table and a pool of exactly len(index) x row-width pages (the reference ABI's pool =
    batch x row width; the pages no sequence uses stay in the pool).  Used for golden
    vectors of the reference's own operator at the benchmark's shapes."""
    cfg = CONFIGS[name]
    L_all, _ = config_seq_lens(name)
    lens = [int(L_all[i]) for i in index]
    P = cfg["P"]
    npg = [(L + P - 1) // P for L in lens]
    width = max(npg)
    spare = len(lens) * width - sum(npg)
    inp = custom_case(len(lens), cfg["Hq"], cfg["Hkv"], P, lens, seed=seed, table="permuted",
                      spare_pages=spare, width=width, std_kv=0.5 if name == "c4" else 1.0)
    inp.name = f"{name}_slice"
    return inp


def golden_slice_index(name):
    """The sequences the golden slices keep: c3 its first 8; c4 its shortest, median,
    90th-percentile and longest (its lengths are log-uniform over [64, 65536])."""
    L_all, _ = config_seq_lens(name)
    if name == "c3":
        return list(range(8))
    order = torch.argsort(L_all.to(torch.int64)).tolist()
    n = len(order)
    return [order[0], order[n // 2], order[(9 * n) // 10], order[-1]]


# --------------------------------------------------------------------------------------
# The reference's correctness table
# --------------------------------------------------------------------------------------

# verify_real.py:8-10 -- case: (batch, seqlen_k capacity, num_heads_k); num_heads = 32.
SPJ_CASES = {1: (1, 1, 4), 2: (4, 2, 8), 3: (16, 17, 4), 4: (64, 64, 8), 5: (16, 141, 4),
             6: (16, 362, 8), 7: (64, 2048, 8), 8: (16, 4096, 4), 9: (32, 4096, 8),
             10: (1, 8192, 4), 11: (16, 12251, 4), 12: (8, 32768, 8), 13: (1, 58966, 8),
             14: (1, 61519, 4)}
EDGE_CASES = (1, 2, 3)


def spj_case(case, table="contiguous", seed=42, device="cpu"):
    """Case `case` of the reference's table, generated like verify_real.py:19-31 but on
    the CPU generator (so the same bytes come out on any machine with this torch)."""
    batch, seq, kv = SPJ_CASES[case]
    nh, D, P = 32, HEAD_DIM, 16
    bpb = math.ceil(seq / P)
    nb = batch * bpb
    torch.manual_seed(seed)
    if case == 1:
        cs = torch.full((batch,), 1, dtype=torch.int32)
    else:
        cs = torch.randint(1, seq + 1, (batch,), dtype=torch.int32)
        cs[0] = seq
        if batch > 1:
            cs[1] = 1
    q = torch.randn(batch, 1, nh, D, dtype=torch.bfloat16)
    k = torch.randn(nb, P, kv, D, dtype=torch.bfloat16)
    v = torch.randn(nb, P, kv, D, dtype=torch.bfloat16)
    if table == "contiguous":
        bt = torch.arange(nb, dtype=torch.int32).reshape(batch, bpb)
    else:
        g = _generator(seed + 7, "cpu")
        bt = torch.randperm(nb, generator=g).to(torch.int32).reshape(batch, bpb)
    inp = DecodeInputs(q=q.view(batch, nh, D), k=k, v=v, block_table=bt, seq_lens=cs,
                       scale=1.0 / math.sqrt(D), name=f"spj{case}", seqlen_k=seq)
    return inp.to(device) if device != "cpu" else inp


def custom_case(B, Hq, Hkv, P, seq_lens, seed=0, table="permuted", spare_pages=0,
                width=None, std_kv=1.0, device="cpu"):
    """Arbitrary shape with given lengths (list or tensor)."""
    seq_lens = torch.as_tensor(seq_lens, dtype=torch.int32)
    npg = [(int(L) + P - 1) // P for L in seq_lens.tolist()]
    if width is None:
        width = max(1, max(npg))
    used = sum(npg) if table == "permuted" else B * width
    num_pages = max(1, used + spare_pages)
    g = _generator(seed, "cpu")
    if table == "contiguous":
        bt = torch.arange(B * width, dtype=torch.int32).reshape(B, width)
    else:
        bt = build_table(seq_lens, P, width, num_pages, g, mode="permuted")
    q = _randn((B, Hq, HEAD_DIM), g, "cpu")
    k = _randn((num_pages, P, Hkv, HEAD_DIM), g, "cpu", std_kv)
    v = _randn((num_pages, P, Hkv, HEAD_DIM), g, "cpu", std_kv)
    inp = DecodeInputs(q=q, k=k, v=v, block_table=bt, seq_lens=seq_lens,
                       scale=1.0 / math.sqrt(HEAD_DIM), name="custom",
                       seqlen_k=width * P)
    return inp.to(device) if device != "cpu" else inp


FP8_MAX = 448.0  # largest finite float8_e4m3fn


def to_fp8(inp: DecodeInputs, k_scale=None, v_scale=None, keep_device=False):
    """The same case with float8_e4m3fn pools: per KV head, element / scale rounded to
    e4m3 (scale = that head's max |x| / 448 unless given).  Returns a new DecodeInputs
    carrying k_scale / v_scale ([Hkv] float32), on the CPU unless `keep_device` (then on
    the pools' device, converted a block of pages at a time)."""
    if not keep_device:
        inp = inp.to("cpu")
    Hkv = inp.num_heads_k
    step = max(1, (1 << 28) // max(1, inp.k[0].numel() * 4))  # ~256 MB of fp32 per block

    def quant(pool, scale):
        if scale is None:
            amax = torch.zeros(Hkv, dtype=torch.float32, device=pool.device)
            for i in range(0, pool.shape[0], step):
                amax = torch.maximum(amax, pool[i:i + step].float().abs().amax(dim=(0, 1, 3)))
            scale = amax.clamp(min=1e-6) / FP8_MAX
        scale = torch.as_tensor(scale, dtype=torch.float32).reshape(-1).expand(Hkv)
        scale = scale.to(pool.device).contiguous()
        y = torch.empty(pool.shape, dtype=torch.float8_e4m3fn, device=pool.device)
        for i in range(0, pool.shape[0], step):
            x = pool[i:i + step].float() / scale.view(1, 1, Hkv, 1)
            y[i:i + step] = x.clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn)
        return y, scale

    k8, ks = quant(inp.k, k_scale)
    v8, vs = quant(inp.v, v_scale)
    return dataclasses.replace(inp, k=k8, v=v8, k_scale=ks, v_scale=vs,
                               name=inp.name + "+fp8")


def dequant(pool, scale):
    """float32 values of an e4m3 pool with per-KV-head factors (test helper)."""
    return pool.float() * scale.float().view(1, 1, -1, 1)


def poison(inp: DecodeInputs, value=float("nan")):
    """Fill every KV slot that a correct kernel must not read with `value`:
    pages no valid block-table entry references (including the targets of padding
    slots) and the slots past seq_len inside each sequence's last page.  FP8 pools get
    the e4m3 NaN pattern (0x7f).  Returns a new DecodeInputs (CPU tensors)."""
    inp = inp.to("cpu")
    if inp.k.dtype == torch.float8_e4m3fn:
        pk = poison(dataclasses.replace(inp, k=inp.k.view(torch.uint8), v=inp.v.view(torch.uint8)),
                    value=0x7F)
        return dataclasses.replace(inp, k=pk.k.view(torch.float8_e4m3fn),
                                   v=pk.v.view(torch.float8_e4m3fn), name=inp.name + "+poison")
    k, v = inp.k.clone(), inp.v.clone()
    P = inp.page_size
    used = torch.zeros(inp.num_pages, dtype=torch.bool)
    tail = []
    for b, L in enumerate(inp.seq_lens.tolist()):
        n = (L + P - 1) // P
        ids = inp.block_table[b, :n].to(torch.int64)
        used[ids] = True
        if L % P:
            tail.append((int(ids[-1]), L % P))
    k[~used] = value
    v[~used] = value
    for pid, r in tail:
        k[pid, r:] = value
        v[pid, r:] = value
    return dataclasses.replace(inp, k=k, v=v, name=inp.name + "+poison")
