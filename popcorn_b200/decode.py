"""Decode-layer composition over the C ABI (the hot path the benchmark runs).

The layer follows the reference's decode-layer template
(Examples/GemmaCLI/Sources/GemmaCLI/Gemma4TextInference.swift:312-436),
restricted to BASELINE's layer list (RMSNorm, QKV matvec, KV-cache write,
GQA flash-decode, o_proj, gated MLP) plus the two residual adds:

    xn   = RMSNorm(x) ; q,k,v = W_qkv xn ; KVCacheWrite(k, v at pos)
    attn = FlashDecoding(q, caches[:pos+1])
    h    = x + W_o attn
    act  = act(W_gate RMSNorm(h)) * (W_up RMSNorm(h))
    out  = h + W_down act

It is encoded as five fused kernels per layer (six launches when the
decode attention splits its keys), each equal to the reference op sequence
with the same rounding points:

    QKVProjection (RMSNorm + matvec + KV write)  -> FlashDecodingRagged
    -> MatmulResidual (o_proj + Add) -> GatedMLP (RMSNorm + gate/up + act*up)
    -> MatmulResidual (down_proj + Add)

The position lives in device memory, so one captured CUDA graph serves
every decode step.
"""
from .api import AttentionMask, FixedScratch, KernelCommandEncoder, Kernels


class LayerShape:
    """Gemma-2-2B-shape layer."""

    def __init__(self, hidden=2304, q_heads=8, kv_heads=4, head_dim=256, ffn=9216, max_ctx=4096, dtype="f16",
                 eps=1e-6, attn_scale=1.0 / 16, activation=0):
        self.H, self.Nq, self.Nkv, self.Hd, self.F = hidden, q_heads, kv_heads, head_dim, ffn
        self.Smax = max_ctx
        self.dtype = dtype
        self.eps = eps
        self.scale = attn_scale
        self.activation = activation  # 0 GeGLU (gelu_tanh), 1 SwiGLU (silu)

    @property
    def weight_params(self):
        H, Nq, Nkv, Hd, F = self.H, self.Nq, self.Nkv, self.Hd, self.F
        return (Nq + 2 * Nkv) * Hd * H + H * Nq * Hd + 2 * F * H + H * F

    @property
    def elem(self):
        return 4 if self.dtype == "f32" else 2

    def kv_bytes(self, ctx):
        return 2 * self.Nkv * ctx * self.Hd * self.elem

    def bytes_per_token(self, ctx):
        """Algorithmic HBM bytes of one layer at context ctx: every weight
        once, K and V of ctx keys once."""
        return self.weight_params * self.elem + self.kv_bytes(ctx)


def _torch_dtype(dt):
    import torch
    return {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}[dt]


class DecodeLayerWeights:
    """Random-init weights N(0, 0.02) and a pre-filled KV cache N(0, 1)."""

    def __init__(self, shape, generator, device="cuda"):
        import torch
        s = shape
        tdt = _torch_dtype(s.dtype)

        def randn(*sz, std=1.0):
            return (torch.randn(*sz, generator=generator, device=device, dtype=torch.float32) * std).to(tdt)

        self.attn_norm = (torch.randn(s.H, generator=generator, device=device) * 0.1).float()
        self.mlp_norm = (torch.randn(s.H, generator=generator, device=device) * 0.1).float()
        self.w_qkv = randn((s.Nq + 2 * s.Nkv) * s.Hd, s.H, std=0.02)
        self.w_o = randn(s.H, s.Nq * s.Hd, std=0.02)
        self.w_gate = randn(s.F, s.H, std=0.02)
        self.w_up = randn(s.F, s.H, std=0.02)
        self.w_down = randn(s.H, s.F, std=0.02)
        self.k_cache = randn(1, s.Nkv, s.Smax, s.Hd)
        self.v_cache = randn(1, s.Nkv, s.Smax, s.Hd)


class DecodeStack:
    """A stack of decode layers with its activations, position and scratch.

    encode_step() enqueues one token through every layer on the encoder's
    stream; `x` holds the token's hidden state on entry and the stack's
    output on exit (it ping-pongs through two buffers).
    """

    def __init__(self, library, shape, n_layers, seed=0, device=0, l2_prefetch=False, fused=False, vocab=0,
                 qk_norm_rope=False, rope_theta=10000.0, norm_add_one=True, kv_early=None):
        """vocab > 0 adds the step's tail: the final RMSNorm fused into the LM
        head GEMV (tied embedding [vocab, H]) into `logits`, then Argmax into
        `token` (int32) — the greedy next token (Argmax.metal).

        qk_norm_rope adds the Gemma-3/4 attention prologue
        (Gemma4TextInference.swift:346-381): per-head RMSNorm of q and the new
        k (weights q_norm / k_norm) and of the new v (no weight), then RoPE of
        q and k with tables over every position (RopeBuildCosSin, built once
        here). The per-op path runs it as one QKNormRope launch after the QKV
        projection; the fused step folds it into the attention items.

        norm_add_one: RMSNorm weights are applied as (1 + w) (Gemma 2 style,
        RMSNorm.swift addOneToWeight) or as w (Gemma 4).

        kv_early: each layer's decode attention gets PC_HINT_KV_EARLY (the
        kernel before it writes only the newest K/V row), so it copies the
        older K/V tiles while that kernel drains (default on;
        POPCORN_KV_EARLY=0 turns it off for comparisons)."""
        import os
        import torch
        if kv_early is None:
            kv_early = os.environ.get("POPCORN_KV_EARLY", "1") == "1"
        self.kv_early = kv_early
        self.norm_add_one = norm_add_one
        self.shape = shape
        self.library = library
        self.vocab = vocab
        self.device = device
        g = torch.Generator(device="cuda:%d" % device)
        g.manual_seed(seed)
        self.layers = self._make_layers(shape, g, n_layers)
        s = shape
        tdt = _torch_dtype(s.dtype)
        dev = "cuda:%d" % device
        self.qk_norm_rope = qk_norm_rope
        if qk_norm_rope:
            for w in self.layers:
                if not hasattr(w, "q_norm"):  # (weights read from an archive bring their own)
                    w.q_norm = (torch.randn(s.Hd, generator=g, device=dev) * 0.1).float()
                    w.k_norm = (torch.randn(s.Hd, generator=g, device=dev) * 0.1).float()
            self.inv_freq = (rope_theta ** (-torch.arange(0, s.Hd, 2, dtype=torch.float32) / s.Hd)).to(dev)
            self.rope_cos = torch.empty(s.Smax, s.Hd // 2, dtype=torch.float32, device=dev)
            self.rope_sin = torch.empty_like(self.rope_cos)
            positions = torch.arange(s.Smax, dtype=torch.int32, device=dev)
            KernelCommandEncoder(library).encode(
                Kernels.RopeBuildCosSin(positions, self.inv_freq, self.rope_cos, self.rope_sin, 1.0))
            torch.cuda.synchronize(dev)
        # One device block holds the step's inputs: the hidden state x, then
        # the position state [pos, pos + 1] (int32) at a 16-byte boundary,
        # so a caller feeds a step with a single host-to-device copy.
        esz = torch.tensor([], dtype=tdt).element_size()
        self.io_pos_offset = (s.H * esz + 15) // 16 * 16
        self.io = torch.zeros(self.io_pos_offset + 16, dtype=torch.uint8, device=dev)
        self.x = self.io[:s.H * esz].view(tdt).view(1, s.H)
        self.x2 = torch.zeros(1, s.H, dtype=tdt, device=dev)
        self.h = torch.zeros(1, s.H, dtype=tdt, device=dev)
        self.q = torch.zeros(1, s.Nq, 1, s.Hd, dtype=tdt, device=dev)
        self.attn = torch.zeros(1, s.Nq, 1, s.Hd, dtype=tdt, device=dev)
        self.act = torch.zeros(1, s.F, dtype=tdt, device=dev)
        # device-resident position state: [pos, pos + 1]
        self.pos_state = self.io[self.io_pos_offset:self.io_pos_offset + 8].view(torch.int32)
        # scratch for the decode attention partials (reused by every layer)
        self.scratch = FixedScratch(64 << 20, device)
        self.l2_prefetch = l2_prefetch
        self.fused = fused
        if vocab:
            self.final_norm = (torch.randn(s.H, generator=g, device=dev) * 0.1).float()
            self.lm_head = (torch.randn(vocab, s.H, generator=g, device=dev, dtype=torch.float32) * 0.02).to(tdt)
            self.logits = torch.zeros(1, vocab, dtype=tdt, device=dev)
            self.token = torch.zeros(1, dtype=torch.int32, device=dev)
        self._kernels = None

    def _make_layers(self, shape, generator, n_layers):
        return [DecodeLayerWeights(shape, generator) for _ in range(n_layers)]

    def kernels(self):
        """The validated kernel objects of one step (built once)."""
        if self._kernels is not None:
            return self._kernels
        if self.fused:
            return self._fused_kernels()
        s = self.shape
        pos = self.pos_state[0:1]
        lens = self.pos_state[1:2]
        ks = []
        cur, nxt = self.x, self.x2
        for i, w in enumerate(self.layers):
            ks.append(Kernels.QKVProjection(cur, w.attn_norm, w.w_qkv, self.q, w.k_cache, w.v_cache, position=pos,
                                            eps=s.eps, add_one_to_weight=self.norm_add_one))
            if self.qk_norm_rope:
                ks.append(Kernels.QKNormRope(self.q, w.k_cache, w.v_cache, w.q_norm, w.k_norm, self.rope_cos,
                                             self.rope_sin, position=pos, eps=s.eps,
                                             add_one_to_weight=self.norm_add_one,
                                             norm_v=True))
            ks.append(Kernels.FlashDecodingRagged(self.q, w.k_cache, w.v_cache, lens, into=self.attn, scale=s.scale,
                                                  mask=AttentionMask.causal))
            if self.kv_early:
                # the kernel before it (QKV projection, or the q/k/v norm +
                # RoPE) writes only the newest K/V row
                ks[-1].set_hint(Kernels.FlashDecodingRagged.HINT_KV_EARLY)
            ks.append(Kernels.MatmulResidual(self.attn.view(1, s.Nq * s.Hd), w.w_o, cur, into=self.h))
            ks.append(Kernels.GatedMLP(self.h, w.w_gate, w.w_up, into=self.act, norm_weight=w.mlp_norm, eps=s.eps,
                                       add_one_to_weight=self.norm_add_one, activation=s.activation))
            ks.append(Kernels.MatmulResidual(self.act, w.w_down, self.h, into=nxt))
            cur, nxt = nxt, cur
        if self.l2_prefetch:
            self._chain_prefetch(ks)
        self.out = cur
        ks += self._tail_kernels()
        self._kernels = ks
        return ks

    def _fused_kernels(self):
        """The whole step as one persistent kernel (Kernels.DecodeStack)."""
        import torch
        from . import _native as N
        from .api import DecodeStackKernel
        s = self.shape
        dev = self.x.device
        rows = [[w.w_qkv.data_ptr(), w.w_o.data_ptr(), w.w_gate.data_ptr(), w.w_up.data_ptr(), w.w_down.data_ptr(),
                 w.attn_norm.data_ptr(), w.mlp_norm.data_ptr(), w.k_cache.data_ptr(), w.v_cache.data_ptr()]
                + ([w.q_norm.data_ptr(), w.k_norm.data_ptr(), self.rope_cos.data_ptr(), self.rope_sin.data_ptr()]
                   if self.qk_norm_rope else [0, 0, 0, 0])
                for w in self.layers]
        self._layer_table = torch.tensor(rows, dtype=torch.int64).to(dev)
        dt = {"f16": 9, "bf16": 10}[s.dtype]
        desc = N.pc_decode_stack_desc(dt, len(self.layers), s.H, s.Nq, s.Nkv, s.Hd, s.F, s.Smax, s.eps, s.scale,
                                      s.activation, int(self.norm_add_one), self._layer_table.data_ptr(),
                                      self.x.data_ptr(),
                                      self.x2.data_ptr(), self.h.data_ptr(), self.q.data_ptr(),
                                      self.attn.data_ptr(), self.act.data_ptr(), self.pos_state.data_ptr(), None, 0,
                                      int(self.qk_norm_rope), int(self.qk_norm_rope),
                                      s.Smax if self.qk_norm_rope else 0)
        nbytes = DecodeStackKernel.workspace_bytes(desc)
        self._workspace = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
        desc.workspace = self._workspace.data_ptr()
        desc.workspace_bytes = nbytes
        k = DecodeStackKernel(desc, keep=(self._layer_table, self._workspace))
        self.out = self.x if len(self.layers) % 2 == 0 else self.x2
        self._kernels = [k] + self._tail_kernels()
        return self._kernels

    def _tail_kernels(self):
        """Final RMSNorm + LM head GEMV + Argmax (when vocab > 0)."""
        if not self.vocab:
            return []
        s = self.shape
        return [Kernels.RMSNormMatmul(self.out, self.final_norm, self.lm_head, into=self.logits, eps=s.eps,
                                      add_one_to_weight=self.norm_add_one),
                Kernels.Argmax(self.logits, self.token)]

    # Bytes of the next operand each kernel pulls into L2 once its own loads
    # are issued (an L2 of 126 MB holds these comfortably).
    PREFETCH_CAP = 16 << 20

    def _chain_prefetch(self, ks):
        """Each kernel warms L2 with the start of the next kernel's operand
        (QKV -> this layer's K/V cache, attention -> W_o, o_proj -> W_gate and
        W_up, gated MLP -> W_down, down_proj -> the next layer's W_qkv), so
        HBM stays busy across kernel boundaries."""
        cap = self.PREFETCH_CAP
        L = len(self.layers)
        for i, w in enumerate(self.layers):
            nxt = self.layers[(i + 1) % L]
            per = len(ks) // L
            qkv, fd, oproj, mlp, down = [ks[per * i + j] for j in (0, per - 4, per - 3, per - 2, per - 1)]
            qkv.set_l2_prefetch(0, w.k_cache).set_l2_prefetch(1, w.v_cache)
            fd.set_l2_prefetch(0, w.w_o)
            oproj.set_l2_prefetch(0, w.w_gate, min(cap, _nbytes(w.w_gate)))
            oproj.set_l2_prefetch(1, w.w_up, min(cap, _nbytes(w.w_up)))
            mlp.set_l2_prefetch(0, w.w_down, min(2 * cap, _nbytes(w.w_down)))
            down.set_l2_prefetch(0, nxt.w_qkv)

    def encoder(self, stream=None):
        return KernelCommandEncoder(self.library, stream=stream, scratch=self.scratch)

    def set_position(self, pos):
        self.pos_state.copy_(self._pos_tensor(pos))

    def _pos_tensor(self, pos):
        import torch
        return torch.tensor([pos, pos + 1], dtype=torch.int32)

    def encode_step(self, encoder):
        encoder.encode(*self.kernels())
        return self.out

    def algorithmic_bytes_per_step(self, ctx):
        lm = self.vocab * self.shape.H * _nbytes(self.x) // self.x.numel() if self.vocab else 0
        return len(self.layers) * self.shape.bytes_per_token(ctx) + lm


class AqLayerWeights:
    """A decode layer whose five weight matrices are affine 4-bit tensors in
    the reference's MLX format (AffineQuantizedTensor.swift: u32-packed
    values, bf16 scale and bias per 64 inputs): random q in 0..15 with
    scales ~0.004 and biases centring each group, so the dequantised weights
    are ~N(0, 0.02)-sized. W_q/W_k/W_v are one [(Nq+2Nkv)*Hd, H] tensor and
    W_gate/W_up one [2F, H] tensor with rows interleaved in blocks of 8 (rows
    16i..16i+7 are gate rows 8i..8i+7, rows 16i+8..16i+15 the up rows), the
    layout the fused gated form reads. Norm weights f32, KV cache bf16
    N(0, 1)."""

    def __init__(self, shape, generator, device="cuda"):
        import torch
        s = shape

        def q4(n, k):
            return _random_q4(n, k, generator, device)

        self.attn_norm = (torch.randn(s.H, generator=generator, device=device) * 0.1).float()
        self.mlp_norm = (torch.randn(s.H, generator=generator, device=device) * 0.1).float()
        self.w_qkv = q4((s.Nq + 2 * s.Nkv) * s.Hd, s.H)
        self.w_o = q4(s.H, s.Nq * s.Hd)
        self.w_gate = q4(s.F, s.H)
        self.w_up = q4(s.F, s.H)
        self.w_gate_up = _interleave8(self.w_gate, self.w_up)
        self.w_down = q4(s.H, s.F)
        self.k_cache = torch.randn(1, s.Nkv, s.Smax, s.Hd, generator=generator, device=device).bfloat16()
        self.v_cache = torch.randn(1, s.Nkv, s.Smax, s.Hd, generator=generator, device=device).bfloat16()

    @staticmethod
    def nbytes(qt):
        n, k = qt.shape
        return n * k // 2 + 2 * n * (k // 64) * 2


def _random_q4(n, k, generator, device):
    """A random 4-bit affine tensor [n, k]: q uniform in 0..15, bf16 scales
    ~0.004 and biases centring each group (dequantised values ~N(0, 0.02))."""
    import torch
    from .api import AffineQuantizedTensor
    packed = torch.randint(-2 ** 31, 2 ** 31 - 1, (n, k // 8), generator=generator, device=device,
                           dtype=torch.int64).to(torch.int32)
    sc = torch.rand(n, k // 64, generator=generator, device=device) * 0.004 + 0.002
    bi = -7.5 * sc + torch.randn(n, k // 64, generator=generator, device=device) * 0.002
    return AffineQuantizedTensor(packed, sc.bfloat16(), bi.bfloat16(), (n, k))


def _interleave8(a, b):
    """[a; b] with rows interleaved in blocks of 8 (a's rows 8i..8i+7, then
    b's), for packed values, scales and biases alike."""
    import torch
    from .api import AffineQuantizedTensor

    def il(x, y):
        n = x.shape[0]
        return torch.stack([x.view(n // 8, 8, -1), y.view(n // 8, 8, -1)], dim=1).reshape(2 * n, -1).contiguous()

    return AffineQuantizedTensor(il(a.packed_tensor, b.packed_tensor), il(a.scales, b.scales),
                                 il(a.biases, b.biases), (2 * a.out_features, a.in_features))


def _concat_rows(ts):
    """Row-wise concatenation of affine 4-bit tensors with one in_features
    (the format's rows are independent: packed values, scales and biases
    concatenate alike)."""
    import torch
    from .api import AffineQuantizedTensor
    return AffineQuantizedTensor(torch.cat([t.packed_tensor for t in ts]).contiguous(),
                                 torch.cat([t.scales for t in ts]).contiguous(),
                                 torch.cat([t.biases for t in ts]).contiguous(),
                                 (sum(t.out_features for t in ts), ts[0].in_features),
                                 bits=ts[0].bits, group_size=ts[0].group_size)


class ArchiveAqLayer:
    """One decode layer's 4-bit weights read through a WeightLoader
    (Gemma4Weights.swift:59-75 names): q/k/v_proj concatenated into w_qkv,
    gate/up_proj kept and interleaved for the fused gated form, norms
    (input_layernorm before attention, pre_feedforward_layernorm before the
    MLP, self_attn.q_norm / k_norm) widened to f32; fresh bf16 KV caches."""

    def __init__(self, loader, index, shape, device):
        import torch
        p = loader.layer_prefix(index)
        lin = loader.linear
        self.w_qkv = _concat_rows([lin(p + ".self_attn.q_proj"), lin(p + ".self_attn.k_proj"),
                                   lin(p + ".self_attn.v_proj")])
        self.w_o = lin(p + ".self_attn.o_proj")
        self.w_gate, self.w_up = lin(p + ".mlp.gate_proj"), lin(p + ".mlp.up_proj")
        self.w_gate_up = _interleave8(self.w_gate, self.w_up)
        self.w_down = lin(p + ".mlp.down_proj")
        self.attn_norm = loader.norm_weight(p + ".input_layernorm.weight")
        self.mlp_norm = loader.norm_weight(p + ".pre_feedforward_layernorm.weight")
        if p + ".self_attn.q_norm.weight" in loader.archive:
            self.q_norm = loader.norm_weight(p + ".self_attn.q_norm.weight")
            self.k_norm = loader.norm_weight(p + ".self_attn.k_norm.weight")
        s = shape
        self.k_cache = torch.zeros(1, s.Nkv, s.Smax, s.Hd, dtype=torch.bfloat16, device=device)
        self.v_cache = torch.zeros_like(self.k_cache)


class AqDecodeStack(DecodeStack):
    """DecodeStack over 4-bit affine weights (bf16 activations): per layer

        xn = RMSNorm(x); qkv = Matmul(xn, W_qkv) -> q, K/V rows (QKVScatter)
        [QKNormRope]; attn = FlashDecoding; o = Matmul(attn, W_o)
        h = x + o, hn = RMSNorm(h) (AddRMSNorm); gu = Matmul(hn, [W_gate; W_up])
        act = act(g) * u (GatedActivation); x' = h + Matmul(act, W_down) (Add)

    — the reference layer (Gemma4TextInference.swift:312-436) with its
    Matmuls on AffineQuantizedTensor weights (Matmul.swift:99-131), every
    intermediate stored in bf16 where the reference stores it."""

    @classmethod
    def from_archive(cls, library, shape, loader, n_layers, **kwargs):
        """The stack over the first n_layers of a 4-bit safetensors archive
        (popcorn_b200.safetensors.WeightLoader)."""
        kwargs["layers"] = [ArchiveAqLayer(loader, i, shape, "cuda:%d" % kwargs.get("device", 0))
                            for i in range(n_layers)]
        return cls(library, shape, n_layers, **kwargs)

    def __init__(self, *args, ops="fused", vocab=0, layers=None, **kwargs):
        """ops="fused": five launches per layer (+ the attention's two) —
        AqQKVProjection (RMSNorm + QKV + KV write), [QKNormRope],
        FlashDecodingRagged, AqMatmulResidual (o_proj + Add), AqGatedMLP
        (RMSNorm + gate/up + act * up), AqMatmulResidual (down_proj + Add).
        ops="reference": the reference's op sequence, one kernel per op.
        vocab > 0: the step's tail on a 4-bit tied embedding [vocab, H]
        (EmbeddingTable.encodeLMHead, EmbeddingTable.swift:38-46): final
        RMSNorm fused into the LM head GEMV, then Argmax into `token`."""
        import torch
        self.ops = ops
        self._given_layers = layers
        super().__init__(*args, **kwargs)
        self.vocab = vocab
        if vocab:
            s = self.shape
            g = torch.Generator(device="cuda:%d" % self.device)
            g.manual_seed(kwargs.get("seed", 0) + 7919)
            dev = self.x.device
            self.final_norm = (torch.randn(s.H, generator=g, device=dev) * 0.1).float()
            self.lm_head = _random_q4(vocab, s.H, g, dev)
            self.logits = torch.zeros(1, vocab, dtype=torch.bfloat16, device=dev)
            self.token = torch.zeros(1, dtype=torch.int32, device=dev)

    def _tail_kernels(self):
        if not self.vocab:
            return []
        s = self.shape
        return [Kernels.AqRMSNormMatmul(self.out, self.final_norm, self.lm_head, self.logits, eps=s.eps,
                                        add_one_to_weight=self.norm_add_one),
                Kernels.Argmax(self.logits, self.token)]

    def _make_layers(self, shape, generator, n_layers):
        assert shape.dtype == "bf16", "the 4-bit stack runs bf16 activations"
        if self._given_layers is not None:
            return self._given_layers
        return [AqLayerWeights(shape, generator) for _ in range(n_layers)]

    def _fused_layer(self, w, cur, nxt, pos, lens):
        s = self.shape
        ks = [Kernels.AqQKVProjection(cur, w.attn_norm, w.w_qkv, self.q, w.k_cache, w.v_cache, position=pos,
                                      eps=s.eps, add_one_to_weight=self.norm_add_one)]
        if self.qk_norm_rope:
            ks.append(Kernels.QKNormRope(self.q, w.k_cache, w.v_cache, w.q_norm, w.k_norm, self.rope_cos,
                                         self.rope_sin, position=pos, eps=s.eps,
                                         add_one_to_weight=self.norm_add_one, norm_v=True))
        ks.append(Kernels.FlashDecodingRagged(self.q, w.k_cache, w.v_cache, lens, into=self.attn, scale=s.scale,
                                              mask=AttentionMask.causal))
        if self.kv_early:
            # the kernel before it writes only the newest K/V row
            ks[-1].set_hint(Kernels.FlashDecodingRagged.HINT_KV_EARLY)
        ks.append(Kernels.AqMatmulResidual(self.attn.view(1, s.Nq * s.Hd), w.w_o, cur, into=self.h))
        ks.append(Kernels.AqGatedMLP(self.h, w.mlp_norm, w.w_gate_up, into=self.act, eps=s.eps,
                                     add_one_to_weight=self.norm_add_one, activation=s.activation))
        ks.append(Kernels.AqMatmulResidual(self.act, w.w_down, self.h, into=nxt))
        return ks

    def kernels(self):
        import torch
        if self._kernels is not None:
            return self._kernels
        s = self.shape
        dev = self.x.device
        pos = self.pos_state[0:1]
        lens = self.pos_state[1:2]
        bf = torch.bfloat16
        self.xn = torch.zeros(1, s.H, dtype=bf, device=dev)
        self.qkv = torch.zeros(1, (s.Nq + 2 * s.Nkv) * s.Hd, dtype=bf, device=dev)
        self.o = torch.zeros(1, s.H, dtype=bf, device=dev)
        self.hn = torch.zeros(1, s.H, dtype=bf, device=dev)
        self.g_out = torch.zeros(1, s.F, dtype=bf, device=dev)
        self.u_out = torch.zeros(1, s.F, dtype=bf, device=dev)
        self.a_out = torch.zeros(1, s.F, dtype=bf, device=dev)
        self.dn = torch.zeros(1, s.H, dtype=bf, device=dev)
        ks = []
        cur, nxt = self.x, self.x2
        for w in self.layers:
            if self.ops == "fused":
                ks += self._fused_layer(w, cur, nxt, pos, lens)
                cur, nxt = nxt, cur
                continue
            ks.append(Kernels.RMSNorm(cur, w.attn_norm, into=self.xn, eps=s.eps, add_one_to_weight=self.norm_add_one))
            ks.append(Kernels.Matmul(self.xn, w.w_qkv, self.qkv))
            ks.append(Kernels.QKVScatter(self.qkv, self.q, w.k_cache, w.v_cache, position=pos))
            if self.qk_norm_rope:
                ks.append(Kernels.QKNormRope(self.q, w.k_cache, w.v_cache, w.q_norm, w.k_norm, self.rope_cos,
                                             self.rope_sin, position=pos, eps=s.eps,
                                             add_one_to_weight=self.norm_add_one,
                                             norm_v=True))
            ks.append(Kernels.FlashDecodingRagged(self.q, w.k_cache, w.v_cache, lens, into=self.attn, scale=s.scale,
                                                  mask=AttentionMask.causal))
            ks.append(Kernels.Matmul(self.attn.view(1, s.Nq * s.Hd), w.w_o, self.o))
            ks.append(Kernels.AddRMSNorm(cur, self.o, w.mlp_norm, self.h, self.hn, eps=s.eps,
                                         add_one_to_weight=self.norm_add_one))
            ks.append(Kernels.Matmul(self.hn, w.w_gate, self.g_out))
            ks.append(Kernels.Matmul(self.hn, w.w_up, self.u_out))
            ks.append(Kernels.GeluTanh(self.g_out, self.a_out) if s.activation == 0 else
                      Kernels.SiLU(self.g_out, self.a_out))
            ks.append(Kernels.Mul(self.a_out, self.u_out, self.act))
            ks.append(Kernels.Matmul(self.act, w.w_down, self.dn))
            ks.append(Kernels.Add(self.h, self.dn, into=nxt))
            cur, nxt = nxt, cur
        self.out = cur
        ks += self._tail_kernels()
        self._kernels = ks
        return ks

    def algorithmic_bytes_per_step(self, ctx):
        per = sum(AqLayerWeights.nbytes(t) for t in (self.layers[0].w_qkv, self.layers[0].w_o,
                                                    self.layers[0].w_gate, self.layers[0].w_up,
                                                    self.layers[0].w_down))
        head = AqLayerWeights.nbytes(self.lm_head) if self.vocab else 0
        return len(self.layers) * (per + self.shape.kv_bytes(ctx)) + head


def _nbytes(t):
    return t.numel() * t.element_size()


__all__ = ["LayerShape", "DecodeLayerWeights", "DecodeStack", "AqLayerWeights", "ArchiveAqLayer", "AqDecodeStack"]
