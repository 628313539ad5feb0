"""Tensor-parallel batched decode over the C ABI.

Gemma-2-9B-shape decoder (hidden 3584, 16 Q / 8 KV heads, head_dim 256, FFN
14336, vocab 256000, 42 layers) at batch 32, one process per GPU. Each rank
holds:

  * Q / K / V projections: the rows of its query heads and KV heads
    (column-parallel: no communication);
  * o_proj: the columns of its query heads (row-parallel: partial sums);
  * gate / up: a contiguous slice of FFN rows (column-parallel);
  * down_proj: the matching slice of FFN columns (row-parallel);
  * the LM head (tied embedding): a contiguous slice of the vocabulary.

After o_proj and after down_proj each rank holds a partial [B, hidden] sum;
one all-reduce (NCCL over NVLink, `torch.distributed`) completes it before
the residual add — two all-reduces per layer. Norms and residual adds are
replicated. KV heads must divide evenly: TP <= 8 for 8 KV heads.

Every computation is a popcorn_b200 kernel (Matmul on the tcgen05 tensor
cores for M = 32, RMSNorm, KVCacheWrite, ragged FlashDecoding, GeluTanh,
Mul, Add); torch provides device memory, streams and the collective.
"""
from .api import AttentionMask, FixedScratch, KernelCommandEncoder, Kernels, PeerGroup


class TPShape:
    def __init__(self, hidden=3584, q_heads=16, kv_heads=8, head_dim=256, ffn=14336, vocab=256000, layers=42,
                 batch=32, ctx=8192, dtype="bf16", eps=1e-6, attn_scale=1.0 / 16):
        self.H, self.Nq, self.Nkv, self.Hd, self.F, self.V = hidden, q_heads, kv_heads, head_dim, ffn, vocab
        self.L, self.B, self.ctx, self.dtype, self.eps, self.scale = layers, batch, ctx, dtype, eps, attn_scale

    def weight_bytes(self, world=1):
        s = self
        per_layer = ((s.Nq + 2 * s.Nkv) * s.Hd * s.H + s.H * s.Nq * s.Hd + 3 * s.F * s.H) * 2
        return (s.L * per_layer + s.V * s.H * 2) // world

    def kv_bytes(self, world=1):
        s = self
        return s.L * 2 * s.B * s.Nkv * s.ctx * s.Hd * 2 // world


def shard_plan(shape, rank, world):
    """Index ranges a rank owns (the same plan the CPU gloo test checks)."""
    s = shape
    if s.Nkv % world or s.Nq % world or s.F % world or s.V % world:
        raise ValueError("heads, FFN and vocab must divide by the TP degree %d" % world)
    nq, nkv, f, v = s.Nq // world, s.Nkv // world, s.F // world, s.V // world
    return {
        "q_heads": (rank * nq, (rank + 1) * nq),
        "kv_heads": (rank * nkv, (rank + 1) * nkv),
        "ffn": (rank * f, (rank + 1) * f),
        "vocab": (rank * v, (rank + 1) * v),
    }


def shard_layer(full, shape, plan):
    """Slices a full layer's weights (numpy or torch, [out, in]) for one rank."""
    s = shape
    q0, q1 = plan["q_heads"]
    k0, k1 = plan["kv_heads"]
    f0, f1 = plan["ffn"]
    return {
        "w_q": full["w_q"][q0 * s.Hd:q1 * s.Hd],
        "w_k": full["w_k"][k0 * s.Hd:k1 * s.Hd],
        "w_v": full["w_v"][k0 * s.Hd:k1 * s.Hd],
        "w_o": full["w_o"][:, q0 * s.Hd:q1 * s.Hd],
        "w_gate": full["w_gate"][f0:f1],
        "w_up": full["w_up"][f0:f1],
        "w_down": full["w_down"][:, f0:f1],
        "attn_norm": full["attn_norm"],
        "mlp_norm": full["mlp_norm"],
    }


class TPDecodeModel:
    """One rank's shard of the config-5 model with its KV cache and buffers.

    step() enqueues one decode token for the whole batch through every layer
    and the LM head; all_reduce(t) is called on each partial sum (NCCL in the
    benchmark). The position (fixed at ctx - 1, every sequence attends to
    ctx keys) makes each step the same work as a real step at that context.

    Per layer (10 launches + 2 all-reduces, or 10 launches with the peer
    all-reduce fused into the add + norm): one Matmul against the
    concatenated [W_q; W_k; W_v] and a QKVScatter (q out, K/V rows into the
    caches); ragged FlashDecoding; o_proj; all-reduce; AddRMSNorm (residual
    add + MLP norm); one Matmul against [W_gate; W_up] and a GatedActivation;
    down_proj; all-reduce; AddRMSNorm (residual add + the next layer's
    attention norm, or the final norm). Each fused op rounds where the
    unfused reference sequence stores.
    """

    def __init__(self, library, shape, rank=0, world=1, seed=0, device=0):
        import torch
        self.s = s = shape
        self.rank, self.world = rank, world
        self.plan = shard_plan(shape, rank, world)
        self.library = library
        dev = "cuda:%d" % device
        dt = {"bf16": torch.bfloat16, "f16": torch.float16}[s.dtype]
        g = torch.Generator(device=dev)
        g.manual_seed(seed * 1000003 + rank)
        self.nq, self.nkv, self.f = nq, nkv, f = s.Nq // world, s.Nkv // world, s.F // world

        def w(*shape_, std=0.02):
            return (torch.randn(*shape_, device=dev, generator=g) * std).to(dt)

        self.layers = []
        for _ in range(s.L):
            self.layers.append({
                "attn_norm": (torch.randn(s.H, device=dev, generator=g) * 0.1).float(),
                "mlp_norm": (torch.randn(s.H, device=dev, generator=g) * 0.1).float(),
                # rows: this rank's q heads, then its K heads, then its V heads
                "w_qkv": w((nq + 2 * nkv) * s.Hd, s.H),
                "w_o": w(s.H, nq * s.Hd),
                # rows: this rank's gate slice, then its up slice
                "w_gu": w(2 * f, s.H),
                "w_down": w(s.H, f),
                "k_cache": w(s.B, nkv, s.ctx, s.Hd, std=1.0), "v_cache": w(s.B, nkv, s.ctx, s.Hd, std=1.0),
            })
        self.final_norm = (torch.randn(s.H, device=dev, generator=g) * 0.1).float()
        self.lm_head = w(s.V // world, s.H)
        B = s.B
        self.x = torch.zeros(B, s.H, device=dev, dtype=dt)
        self.xn = torch.zeros_like(self.x)
        self.h = torch.zeros_like(self.x)
        self.o = torch.zeros_like(self.x)
        self.qkv = torch.zeros(B, (nq + 2 * nkv) * s.Hd, device=dev, dtype=dt)
        self.q = torch.zeros(B, nq, 1, s.Hd, device=dev, dtype=dt)
        self.attn = torch.zeros(B, nq, 1, s.Hd, device=dev, dtype=dt)
        self.gu = torch.zeros(B, 2 * f, device=dev, dtype=dt)
        self.act = torch.zeros(B, f, device=dev, dtype=dt)
        self.logits = torch.zeros(B, s.V // world, device=dev, dtype=dt)
        self.lens = torch.full((B,), s.ctx, device=dev, dtype=torch.int32)
        self.scratch = FixedScratch(64 << 20, device)
        self.device = device
        self.peer = None
        self._ks = None

    def use_peer_allreduce(self, all_gather, fuse_gemm=False):
        """Switches the two all-reduces per layer from the caller's collective
        to the one-shot peer-memory kernel fused with Add + RMSNorm
        (Kernels.AllReduceAddRMSNorm). `all_gather(bytes) -> [bytes]` exchanges
        the IPC handles once (every rank calls this together). With
        fuse_gemm the o_proj / down GEMM and the all-reduce are one kernel
        (Kernels.MatmulAllReduceAddRMSNorm); at batch 32 that measured slower
        (TP2 2145 vs 2229 tok/s: the GEMM's grid waits on the peers instead
        of letting the next kernel start), so it is off by default."""
        s = self.s
        self.peer = PeerGroup(self.device, self.world, self.rank, s.B, s.H, s.dtype, all_gather)
        self.fuse_gemm = fuse_gemm
        self._ks = None

    def kernels(self):
        """Kernel objects of one step in order; None marks an all-reduce of
        self.o (the partial o_proj / down_proj sum)."""
        if self._ks is not None:
            return self._ks
        s, K = self.s, Kernels
        peer = self.peer
        o_a = peer.partial(0) if peer else self.o  # o_proj partial sum
        o_b = peer.partial(1) if peer else self.o  # down_proj partial sum

        fuse = peer is not None and getattr(self, "fuse_gemm", False) and s.B <= 64

        def gemm_reduce_add_norm(a, w, buf, part, residual, weight, sum_out):
            """The partial-sum GEMM and its all-reduce + Add + RMSNorm: one
            kernel (fused), GEMM + peer kernel, or GEMM + collective + AddRMSNorm."""
            if fuse:
                return [K.MatmulAllReduceAddRMSNorm(a, w, peer, buf, residual, weight, sum_out, self.xn, eps=s.eps,
                                                    add_one_to_weight=True)]
            ks = [K.Matmul(a, w, into=part, transpose_b=True)]
            if peer:
                return ks + [K.AllReduceAddRMSNorm(peer, buf, residual, weight, sum_out, self.xn, eps=s.eps,
                                                   add_one_to_weight=True)]
            return ks + [None, K.AddRMSNorm(residual, part, weight, sum_out, self.xn, eps=s.eps,
                                            add_one_to_weight=True)]

        ks = [K.RMSNorm(self.x, self.layers[0]["attn_norm"], into=self.xn, eps=s.eps, add_one_to_weight=True)]
        for i, w in enumerate(self.layers):
            nxt_norm = self.layers[i + 1]["attn_norm"] if i + 1 < len(self.layers) else self.final_norm
            ks += [K.Matmul(self.xn, w["w_qkv"], into=self.qkv, transpose_b=True),
                   K.QKVScatter(self.qkv, self.q, w["k_cache"], w["v_cache"], offset=s.ctx - 1),
                   K.FlashDecodingRagged(self.q, w["k_cache"], w["v_cache"], self.lens, into=self.attn,
                                         scale=s.scale, mask=AttentionMask.causal)]
            ks += gemm_reduce_add_norm(self.attn.view(s.B, self.nq * s.Hd), w["w_o"], 0, o_a, self.x, w["mlp_norm"],
                                       self.h)
            ks += [K.Matmul(self.xn, w["w_gu"], into=self.gu, transpose_b=True),
                   K.GatedActivation(self.gu, self.act)]
            ks += gemm_reduce_add_norm(self.act, w["w_down"], 1, o_b, self.h, nxt_norm, self.x)
        ks += [K.Matmul(self.xn, self.lm_head, into=self.logits, transpose_b=True)]
        self._ks = ks
        return ks

    def encoder(self, stream=None):
        return KernelCommandEncoder(self.library, stream=stream, scratch=self.scratch)

    def step(self, encoder, all_reduce):
        for k in self.kernels():
            if k is None:
                all_reduce(self.o)
            else:
                encoder.encode(k)

    def bytes_per_step(self):
        """Algorithmic HBM bytes one rank moves per step: its weight shard
        once and its KV-cache shard once."""
        return self.s.weight_bytes(self.world) + self.s.kv_bytes(self.world)


__all__ = ["TPShape", "TPDecodeModel", "shard_plan", "shard_layer"]
