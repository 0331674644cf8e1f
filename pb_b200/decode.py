"""Harness of one decode step of a synthetic MLA + MoE model (BASELINE config
4), standing in for the reference runtime's Rust layer loop
(forward_token_input, runtime/mod.rs:1432-2024), which stays in the
reference: this module allocates the step's buffers with torch and enqueues the
C-ABI calls a Rust host would make per layer, so the benchmark and the tests
can run the whole step. Python only enqueues; every operation is a CUDA kernel
behind pbmoe_*; `DecodeStep.launch` is what a CUDA graph captures.

Per layer, with the GLM MLA attention of mla_attention_output_values
(runtime/mod.rs:2779-2940):

  qa, kv = Q4(q_a_proj) xn, Q4(kv_a_proj_with_mqa) xn            pbmoe_q4_matvec_fused (2 matrices)
  q      = Q4(q_b_proj) rms_norm(qa) w_qa                         pbmoe_q4_matvec_fused (input norm)
  RoPE on q's and kv's rope parts; rms_norm(kv[:latent]) w_kv,
  the rotated key written into the caches, then
  attn   = absorbed MLA attention over the cache                  pbmoe_mla_append_decode (latent norm)
  h      = x + Q4(o_proj) attn                                    pbmoe_q4_matvec_fused (residual)
  x      = h + MoE(rms_norm(h) w_post), xn = rms_norm(x) w_in'    pbmoe_moe_layer (input norm, next norm)

and after the last layer (whose fused norm uses the final norm weight) the
vocab head top-k (pbmoe_head_topk). The residual stream x is f32; the MLA
projection inputs are f32; caches are bf16 per (layer, sequence).

The projection shapes (q_lora 1536, kv_a 512 + 64, q_b 16 x 192, o_proj 16 x
128 -> hidden) are this build's declaration for config 4, which fixes only the
attention geometry (16 heads, nope 128, rope 64, latent 512, v 128): they are
GLM-style 4-bit group-64 projections as in the reference's GLM path.
"""

from __future__ import annotations

from dataclasses import dataclass

import contextlib

import torch

from . import capi, synth


def _null():
    return contextlib.nullcontext()


@dataclass
class StepConfig:
    hidden: int = 2048
    layers: int = 48
    q_lora: int = 1536
    heads: int = 16
    nope: int = 128
    rope: int = 64
    latent: int = 512
    v_dim: int = 128
    experts: int = 512
    top_k: int = 10
    inter: int = 512
    group: int = 64
    vocab: int = 151936
    context: int = 8192
    theta: float = 10000.0
    eps: float = 1e-6
    candidates: int = 64  # head top-k


class Q4:
    """A dense Q4 projection [rows x cols] (nibbles, bf16 scales and biases)."""

    def __init__(self, rows, cols, group, g, device):
        self.rows, self.cols, self.group = rows, cols, group
        self.packed, self.scales, self.biases = synth.q4_matrix(rows, cols, group, g, device)

    def mat(self):
        return (self.packed, self.scales, self.biases, self.rows, self.cols, self.group)

    def __call__(self, ctx, x, y, stream):
        ctx.q4_matvec(self.packed, self.scales, self.biases, self.rows, self.cols, self.group, x, y,
                      batch=int(x.shape[0]), stream=stream)

    def nbytes(self):
        return int(self.packed.numel() + 2 * self.scales.numel() + 2 * self.biases.numel())


class Layer:
    """One layer's weights. With `experts` = (begin, count) only that expert
    shard is kept (every rank generates the same full table from the same seed
    and keeps its slots), and `shared` says whether this rank holds the shared
    expert and its gate (expert parallelism: exactly one rank does)."""

    def __init__(self, cfg: StepConfig, seed: int, device="cuda", experts=None, shared=True):
        g = synth.gen(device, seed)
        H, G = cfg.hidden, cfg.group
        self.q_a = Q4(cfg.q_lora, H, G, g, device)
        self.kv_a = Q4(cfg.latent + cfg.rope, H, G, g, device)
        self.q_b = Q4(cfg.heads * (cfg.nope + cfg.rope), cfg.q_lora, G, g, device)
        self.o_proj = Q4(H, cfg.heads * cfg.v_dim, G, g, device)
        norm = lambda n: (1.0 + 0.1 * torch.randn(n, generator=g, device=device)).float()
        self.q_a_norm, self.kv_a_norm = norm(cfg.q_lora), norm(cfg.latent)
        self.input_norm, self.post_norm = norm(H), norm(H)
        self.w_uk = synth.normal_bf16((cfg.heads, cfg.nope, cfg.latent), 0.02, g, device)
        self.w_uv = synth.normal_bf16((cfg.heads, cfg.v_dim, cfg.latent), 0.02, g, device)
        self.moe = synth.MoeLayerWeights(device, seed + 7919, hidden=H, num_experts=cfg.experts,
                                         intermediate=cfg.inter, group=G)
        if experts is not None:
            b, n = experts
            self.moe.experts = self.moe.experts[b:b + n].clone()
            if not shared:
                self.moe.shared, self.moe.shared_gate = None, None
            torch.cuda.empty_cache()

    def nbytes(self):
        """Weight bytes a decode step reads for this layer, before experts."""
        return (self.q_a.nbytes() + self.kv_a.nbytes() + self.q_b.nbytes() + self.o_proj.nbytes() +
                2 * (self.w_uk.numel() + self.w_uv.numel()) +
                4 * (self.q_a_norm.numel() + self.kv_a_norm.numel() + self.input_norm.numel() +
                     self.post_norm.numel()))


class Model:
    """The synthetic model. With ep = (rank, world) this rank keeps expert
    shard rank of every layer (the shared expert on rank 0) and vocabulary
    shard rank of the head (rows [head_base, head_base + head rows)), the
    expert- and vocabulary-parallel layout of a multi-GPU step."""

    def __init__(self, cfg: StepConfig, seed=0, device="cuda", ep=None):
        from . import ep as ep_host

        self.cfg = cfg
        rank, world = ep if ep is not None else (0, 1)
        self.rank, self.world = rank, world
        self.expert_range = capi.ep_expert_range(cfg.experts, rank, world) if ep is not None else None
        self.layers = [Layer(cfg, seed + 1000 * i, device, experts=self.expert_range, shared=rank == 0)
                       for i in range(cfg.layers)]
        g = synth.gen(device, seed + 17)
        self.head = synth.normal_bf16((cfg.vocab, cfg.hidden), 0.02, g, device)
        self.final_norm = (1.0 + 0.1 * torch.randn(cfg.hidden, generator=g, device=device)).float()
        self.head_base = 0
        if ep is not None:
            self.head_base, rows = ep_host.vocab_ranges(cfg.vocab, world)[rank]
            self.head = self.head[self.head_base:self.head_base + rows].clone()
            torch.cuda.empty_cache()


class Caches:
    """bf16 latent and rotated-key caches per (layer, sequence), [context x dim]."""

    def __init__(self, cfg: StepConfig, batch: int, seed=0, device="cuda"):
        g = synth.gen(device, seed + 29)
        self.c_kv = [[synth.normal_bf16((cfg.context, cfg.latent), 1.0, g, device) for _ in range(batch)]
                     for _ in range(cfg.layers)]
        self.k_rope = [[synth.normal_bf16((cfg.context, cfg.rope), 1.0, g, device) for _ in range(batch)]
                       for _ in range(cfg.layers)]
        self.c_kv_ptrs = [torch.tensor([t.data_ptr() for t in l], dtype=torch.int64, device=device)
                          for l in self.c_kv]
        self.k_rope_ptrs = [torch.tensor([t.data_ptr() for t in l], dtype=torch.int64, device=device)
                            for l in self.k_rope]


class DecodeStep:
    """Buffers and launch sequence of one decode step for `batch` sequences,
    each at position positions[b] of its caches (attending over positions
    0..position)."""

    def __init__(self, ctx: capi.Context, model: Model, caches: Caches, batch: int, positions):
        cfg = model.cfg
        self.ctx, self.model, self.caches, self.cfg, self.B = ctx, model, caches, cfg, batch
        dev = "cuda"
        f32 = dict(device=dev, dtype=torch.float32)
        self.positions_host = [int(p) for p in positions]
        self.positions = torch.tensor(self.positions_host, dtype=torch.int32, device=dev)
        B, H = batch, cfg.hidden
        self.x = torch.zeros(B, H, **f32)        # residual stream
        self.xn = torch.zeros(B, H, **f32)       # normed layer input
        self.qa = torch.zeros(B, cfg.q_lora, **f32)
        self.kv = torch.zeros(B, cfg.latent + cfg.rope, **f32)
        self.q = torch.zeros(B, cfg.heads, cfg.nope + cfg.rope, **f32)
        self.attn = torch.zeros(B, cfg.heads, cfg.v_dim, **f32)
        self.o = torch.zeros(B, H, **f32)
        self.h = torch.zeros(B, H, **f32)
        self.n = torch.zeros(B, H, device=dev, dtype=torch.bfloat16)  # normalised MoE input (recorded only)
        self.logits = torch.zeros(B, cfg.vocab, **f32)  # head logits (recorded only)
        self.route_ids = torch.zeros(cfg.layers, B, cfg.top_k, device=dev, dtype=torch.int32)
        self.ids = torch.zeros(B, cfg.candidates, device=dev, dtype=torch.int32)
        self.vals = torch.zeros(B, cfg.candidates, **f32)
        self.mla_cfg = capi.mla_config(cfg.heads, cfg.nope, cfg.rope, cfg.latent, cfg.v_dim)
        self.moe_cfg = capi.moe_config(model.layers[0].moe.layout, cfg.experts, cfg.top_k)
        self.ep = model.expert_range is not None
        self.shard = capi.EpShard(model.expert_range[0], model.expert_range[1], 0) if self.ep else None
        K = cfg.candidates
        # this rank's candidate lists (vocabulary shard) and, under expert
        # parallelism, every rank's after the all-gather
        self.keys = torch.zeros(B, K, device=dev, dtype=torch.int32)
        self.lids = torch.zeros(B, K, device=dev, dtype=torch.int32)
        self.lvals = torch.zeros(B, K, **f32)
        self.gathered = torch.zeros(model.world, 3, B, K, device=dev, dtype=torch.int32) if self.ep else None
        self.moe_w = []
        for l in model.layers:  # the post-attention norm runs inside the MoE layer's router kernel
            w = l.moe.c_weights()
            w.input_norm_weight = l.post_norm.data_ptr()
            self.moe_w.append(w)
        ctx.reserve(B, self.moe_cfg)
        if self.ep:
            from . import ep as ep_host

            ep_host.connect(ctx, max_tokens=B, hidden=H)
        ctx.mla_reserve(self.mla_cfg, B)
        ctx.rope_reserve(cfg.context, cfg.rope, cfg.theta)
        ctx.head_reserve(B, cfg.vocab, cfg.candidates)

    def set_input(self, x):
        """x f32 [B, hidden]: the step's embeddings (residual stream)."""
        self.x.copy_(x)

    def launch(self, stream=None, record_routes=False, record=None, mark=None, moe_events=None):
        """Enqueue the step (under expert parallelism: up to this rank's
        vocabulary-shard candidates; `finish` merges every rank's).
        record_routes writes every layer's route ids to self.route_ids (for
        counting the experts a step reads); record (a dict) receives per-layer
        copies of the intermediates for parity checks (they are copied on the
        current stream: launch on it). mark(name), when given, is called before
        each C-ABI call and once at the end (per-call timing with events);
        moe_events(i) may return the MoE layer's phase-event array for layer i."""
        ctx, cfg, m = self.ctx, self.cfg, self.model
        mk = mark if mark is not None else (lambda name: None)
        L0 = m.layers[0]
        mk("input_norm")
        ctx.rms_norm(self.x, L0.input_norm, self.xn, eps=cfg.eps, stream=stream)
        seq_lens = [p + 1 for p in self.positions_host]
        for i, L in enumerate(m.layers):
            if record is not None:
                record.setdefault("x", []).append(self.x.clone())
                record.setdefault("xn", []).append(self.xn.clone())
            mk("q_a+kv_a")
            ctx.q4_fused([L.q_a.mat(), L.kv_a.mat()], self.xn, [self.qa, self.kv], stream=stream)
            mk("q_b")
            ctx.q4_fused([L.q_b.mat()], self.qa, [self.q.view(self.B, -1)], norm=L.q_a_norm, eps=cfg.eps,
                         stream=stream)
            if record is not None:
                record.setdefault("qa", []).append(self.qa.clone())
                record.setdefault("kv", []).append(self.kv.clone())
                record.setdefault("q_prerope", []).append(self.q.clone())
            mk("mla_decode")  # the RoPE + cache append runs inside the decode's first kernel
            ctx.mla_append_decode(self.mla_cfg, self.q, self.kv, self.positions, self.caches.c_kv_ptrs[i],
                                  self.caches.k_rope_ptrs[i], cfg.context,
                                  [t[:n] for t, n in zip(self.caches.c_kv[i], seq_lens)],
                                  [t[:n] for t, n in zip(self.caches.k_rope[i], seq_lens)], L.w_uk, L.w_uv, self.attn,
                                  latent_norm=L.kv_a_norm, eps=cfg.eps, stream=stream)
            mk("o_proj")
            ctx.q4_fused([L.o_proj.mat()], self.attn.view(self.B, -1), [self.h], residual=self.x, stream=stream)
            if record is not None:
                record.setdefault("q", []).append(self.q.clone())
                record.setdefault("attn", []).append(self.attn.clone())
                record.setdefault("h", []).append(self.h.clone())
            nxt = m.layers[i + 1].input_norm if i + 1 < len(m.layers) else m.final_norm
            dbg = None
            ev = moe_events(i) if moe_events is not None else None
            if record_routes or record is not None or ev is not None:
                dbg = capi.MoeDebug(None, self.route_ids[i].data_ptr() if (record_routes or record is not None)
                                    else None, None, None, ev, self.n.data_ptr() if record is not None else None)
            mk("moe_layer")
            if self.ep:
                if dbg is not None:
                    dbg.phase_events = None
                ctx.ep_moe_layer(self.moe_cfg, self.moe_w[i], self.shard, self.h, self.x, self.B, residual=self.h,
                                 next_norm_weight=nxt, next_normed=self.xn, debug=dbg, stream=stream)
            else:
                ctx.moe_layer(self.moe_cfg, self.moe_w[i], self.h, self.x, self.B, residual=self.h,
                              next_norm_weight=nxt, next_normed=self.xn, debug=dbg, stream=stream)
            if record is not None:
                record.setdefault("n", []).append(self.n.clone())
                record.setdefault("route_ids", []).append(self.route_ids[i].clone())
        mk("head")
        if record is not None:
            record["x_final"] = self.x.clone()
            record["xn_final"] = self.xn.clone()
            ctx.head_topk(m.head, self.xn, self.ids, self.vals, logits=self.logits, stream=stream)
        elif self.ep:
            ctx.head_topk(m.head, self.xn, self.lids, self.lvals, id_base=m.head_base, keys=self.keys,
                          stream=stream)
        else:
            ctx.head_topk(m.head, self.xn, self.ids, self.vals, stream=stream)
        mk("end")

    def finish(self, stream=None):
        """Under expert parallelism: all-gather every rank's vocabulary-shard
        candidate lists (one NCCL collective, ranks in id order) and merge them
        into self.ids / self.vals (pbmoe_head_merge). Nothing on one GPU."""
        if not self.ep:
            return
        import torch.distributed as dist

        local = torch.stack([self.keys, self.lids, self.lvals.view(torch.int32)])
        with torch.cuda.stream(stream) if stream is not None else _null():
            dist.all_gather_into_tensor(self.gathered, local.unsqueeze(0).contiguous())
            g = self.gathered
            self.ctx.head_merge(g[:, 0].contiguous(), g[:, 1].contiguous(), g[:, 2].contiguous().view(torch.float32),
                                self.ids, self.vals, stream=stream)

    def step_weight_bytes(self):
        """Weight bytes one step reads on this rank before routed experts:
        every layer's MLA projections, W_UK/W_UV, norms, router, shared gate
        and shared expert (when this rank holds it), and the head shard."""
        cfg, m = self.cfg, self.model
        L0 = m.layers[0]
        shared = L0.moe.shared is not None
        per_layer = (L0.nbytes() + cfg.experts * cfg.hidden * 2 + (cfg.hidden * 2 if shared else 0) +
                     (int(L0.moe.layout.expert_bytes) if shared else 0))
        return cfg.layers * per_layer + int(m.head.numel()) * 2

    def launches_per_step(self):
        """CUDA kernels one step launches: the input norm; per layer 2 fused
        projection launches, 3 MLA kernels (the first also doing RoPE and the
        cache append), the o_proj launch and 4 MoE kernels per MoE launch
        (one for up to 32 tokens, then one per 32-token chunk); the head's 3
        (plus a memset)."""
        chunks = 1 if self.B <= 8 else (self.B + 31) // 32
        return 1 + self.cfg.layers * (2 + 3 + 1 + 4 * chunks) + 3

    def unique_experts(self):
        """Distinct routed experts per layer in the recorded routes (mean over layers)."""
        ids = self.route_ids.cpu()
        return sum(len(set(ids[i].reshape(-1).tolist())) for i in range(self.cfg.layers)) / self.cfg.layers

    def bytes_per_step(self, unique_experts: float):
        """Algorithmic bytes of one step: every weight byte read once (MLA
        projections, absorbed W_UK/W_UV, norms, router, shared gate, shared
        expert and `unique_experts` routed experts per layer), the cache rows
        attended, the activations in and out, and the vocab head."""
        cfg = self.cfg
        slot = self.model.layers[0].moe.layout.expert_bytes
        per_layer = (self.model.layers[0].nbytes() + cfg.experts * cfg.hidden * 2 + cfg.hidden * 2 +
                     (1 + unique_experts) * slot)
        kv = sum(p + 1 for p in self.positions_host) * (cfg.latent + cfg.rope) * 2
        return int(cfg.layers * (per_layer + kv) + cfg.vocab * cfg.hidden * 2 + self.B * cfg.hidden * 4)
