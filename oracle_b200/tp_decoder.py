"""The hybrid decoder with its heads sharded over the GPUs of one node.

One process per GPU.  Oracle decodes on one CPU thread
(src/runtime/qwen35_block.cpp:406-756, qwen35_forward.cpp:400-470); here rank
q of N (1, 2, 4 or 8) holds and computes only its own heads:

* Gated DeltaNet blocks: its value heads (with the key heads they read), i.e.
  the rows of attn_qkv / attn_gate / ssm_beta / ssm_alpha for those heads,
  their conv channels, decay and time-step entries, recurrent states and conv
  history;
* attention blocks: its query heads (attn_q rows: query and gate of each
  head) and the KV heads those read (attn_k / attn_v rows and the KV cache);
* the MLP: its share of the FFN columns (ffn_gate / ffn_up rows);
* the LM head: a contiguous 1/N of the vocabulary rows.

The two projections whose input is sharded -- the block output projection
(over the heads) and ffn_down (over the FFN columns) -- are computed as
PARTIAL sums: the activation is cut into 256-wide Q8_K blocks and rank q owns
block j of every 16-block segment when j % N == q, so its partial sum of a
row is exactly the subtree of the canonical Q8_K combine order (leaves folded
by strides 8, 4, 2, 1) over its own leaves.  Those partials go to every
rank's gather buffer over NVLink from inside the matvec program, and the next
op's transform folds the N partials by the remaining strides, adds the
segments and the residual, and applies the next RMSNorm -- so every rank
holds the unsharded decoder's hidden vector bit for bit.  The head
assignment follows from the block assignment: a block covers two 128-wide
heads, the key head of value head h is h % key_heads, and the KV head of
query head g is g // (heads / kv_heads); the plan checks that each local head
maps to its local key / KV head by the same rules, so the unchanged
block-core kernels run on the local heads.

Cross-rank dependencies: two per block (after the output projection's
partials, after ffn_down's partials) plus one for the LM head's rows, each
one announcement per rank (oracle_cuda_matvec_program_sharded).  Everything
else -- norms, the residual stream, embedding, sampling -- runs on every rank
on whole vectors, so every rank produces the same tokens.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import FLAG_BUILD_IN_KERNEL, FLAG_PDL, TYPE_F32, TYPE_Q4_K, TYPE_Q6_K, XFORM_COMBINE_RMS, XFORM_RMS, Context
from .qwen35 import Qwen35Config
from .synth import row_bytes

SEGMENT = 16  # Q8_K blocks per segment of the canonical combine order
BLOCK = 256   # elements per Q8_K block


def owned_blocks(n_blocks: int, world: int, rank: int) -> list:
    """The 256-wide blocks of an n_blocks-block vector rank `rank` owns: block
    j of each 16-block segment with j % world == rank (segment-major)."""
    out = []
    for g in range((n_blocks + SEGMENT - 1) // SEGMENT):
        real = min(SEGMENT, n_blocks - g * SEGMENT)
        if real % world:
            raise ValueError(f"{real} blocks in a segment do not split over {world} ranks")
        out += [g * SEGMENT + j for j in range(rank, real, world)]
    return out


@dataclass
class ShardPlan:
    """Which heads, blocks and rows rank `rank` of `world` owns."""
    world: int
    rank: int
    value_heads: list      # Gated DeltaNet value heads (global indices, local order)
    key_heads: list        # the key heads they read (local order)
    q_heads: list          # attention query heads
    kv_heads: list         # the KV heads they read
    ffn_blocks: list       # FFN activation blocks (segment-major)
    ffn_segments: int      # 16-block segments of the FFN activation
    vocab_lo: int
    vocab_hi: int

    @staticmethod
    def make(cfg: Qwen35Config, world: int, rank: int) -> "ShardPlan":
        if world not in (1, 2, 4, 8) or not 0 <= rank < world:
            raise ValueError("world must be 1, 2, 4 or 8 and 0 <= rank < world")
        D = cfg.state_size
        if cfg.head_dim != D or BLOCK % D:
            raise ValueError("head sharding needs 128-wide heads of both kinds")
        per = BLOCK // D  # heads per block
        vh = [per * b + e for b in owned_blocks(cfg.value_width // BLOCK, world, rank) for e in range(per)]
        kh = []
        for h in vh:
            if h % cfg.key_heads not in kh:
                kh.append(h % cfg.key_heads)
        for l, h in enumerate(vh):  # the block core reads key head (local index) l % len(kh)
            if kh[l % len(kh)] != h % cfg.key_heads:
                raise ValueError("value heads do not map to local key heads by h % key_heads")
        qh = [per * b + e for b in owned_blocks(cfg.q_width // BLOCK, world, rank) for e in range(per)]
        group = cfg.heads // cfg.kv_heads
        kv = []
        for g in qh:
            if g // group not in kv:
                kv.append(g // group)
        if len(qh) % len(kv):
            raise ValueError("query heads do not split evenly over their KV heads")
        lg = len(qh) // len(kv)
        for l, g in enumerate(qh):  # the attention kernels read KV head (local) l // lg
            if kv[l // lg] != g // group:
                raise ValueError("query heads do not map to local KV heads in groups")
        fb = owned_blocks(cfg.ffn // BLOCK, world, rank)
        if cfg.vocab % world:
            raise ValueError("the vocabulary does not split evenly")
        v = cfg.vocab // world
        return ShardPlan(world, rank, vh, kh, qh, kv, fb, (cfg.ffn // BLOCK + SEGMENT - 1) // SEGMENT,
                         rank * v, (rank + 1) * v)

    def ffn_segment_blocks(self, g: int) -> list:
        return [b for b in self.ffn_blocks if b // SEGMENT == g]


def _ranges(units: list, width: int) -> np.ndarray:
    """Row (or element) indices of units of `width` consecutive rows."""
    return np.concatenate([np.arange(u * width, (u + 1) * width) for u in units]) if units else np.zeros(0, np.int64)


def take_rows(data: np.ndarray, qtype: int, dims: tuple, rows: np.ndarray) -> np.ndarray:
    """The given rows of a GGML matrix (dims = (cols, rows)), in order."""
    rb = row_bytes(qtype, dims[0])
    return np.ascontiguousarray(data.reshape(dims[1], rb)[rows]).reshape(-1)


def take_blocks(data: np.ndarray, qtype: int, dims: tuple, blocks: list) -> np.ndarray:
    """Every row of a Q4_K / Q6_K matrix restricted to the given 256-column
    blocks (super-blocks), in order: the rows of a column shard."""
    if qtype not in (TYPE_Q4_K, TYPE_Q6_K):
        raise ValueError("column shards of Q4_K / Q6_K matrices only")
    bb = row_bytes(qtype, BLOCK)
    m = data.reshape(dims[1], dims[0] // BLOCK, bb)
    return np.ascontiguousarray(m[:, blocks, :]).reshape(-1)


class HeadShardedDecoder:
    """Rank `rank` of `world` GPUs decoding ONE sequence together with the
    other ranks (one process each; every rank makes the same calls).

    tensors: [(name, ggml type, gguf dims, uint8 bytes)] of the whole model,
    as for ``Qwen35Decoder`` (Q8_K contract: Q4_K / Q6_K matrices); each rank
    uploads its own slices.  exchange(handle) -> every rank's peer-group
    handle, in rank order (e.g. an all_gather_object)."""

    def __init__(self, ctx: Context, cfg: Qwen35Config, tensors, rank: int, world: int, exchange,
                 capacity: int | None = None, max_new: int = 4096, device: int = 0):
        import torch

        from . import PeerGroup
        self.torch, self.ctx, self.cfg = torch, ctx, cfg
        self.rank, self.world = rank, world
        self.plan = plan = ShardPlan.make(cfg, world, rank)
        self.dev = dev = torch.device("cuda", device)
        self.cap = int(capacity or cfg.context)
        self.max_new = int(max_new)
        by_name = {name: (int(qt), tuple(dims), np.ascontiguousarray(data).view(np.uint8).reshape(-1))
                   for name, qt, dims, data in tensors}
        for name, (qt, dims, _) in by_name.items():
            if len(dims) == 2 and qt not in (TYPE_F32, TYPE_Q4_K, TYPE_Q6_K) and name != "token_embd.weight":
                raise ValueError(f"{name}: the Q8_K contract runs Q4_K / Q6_K matrices only")
        self.w = {}
        self._load(by_name)
        H, D, G = cfg.hidden, cfg.state_size, plan.ffn_segments
        f32 = lambda n: torch.zeros(max(int(n), 1), dtype=torch.float32, device=dev)  # noqa: E731
        # gather buffer: every rank's partial sums of the two sharded
        # projections and the logits, 16-byte aligned pieces
        pieces = dict(part_out=world * H, part_down=world * G * H, logits=cfg.vocab)
        sizes = {k: (n + 3) // 4 * 4 for k, n in pieces.items()}
        self.group = PeerGroup(ctx, rank, world, sum(sizes.values()) * 4)
        self.group.connect(exchange(self.group.handle))
        data, off = self.group.tensor(), 0
        for k, n in pieces.items():
            setattr(self, k, data[off:off + n])
            off += sizes[k]
        self.hidden, self.resid = f32(H), f32(H)
        nv, nk, nq, nkv = len(plan.value_heads), len(plan.key_heads), len(plan.q_heads), len(plan.kv_heads)
        self.channels = (2 * nk + nv) * D
        self.qkv, self.z, self.gated = f32(self.channels), f32(nv * D), f32(nv * D)
        self.beta, self.alpha = f32(nv), f32(nv)
        self.q_full, self.k, self.v = f32(2 * nq * D), f32(nkv * D), f32(nkv * D)
        self.qn, self.attn, self.scores = f32(nq * D), f32(nq * D), f32(nq * self.cap)
        nf = len(plan.ffn_blocks) * BLOCK
        self.gate, self.up, self.act = f32(nf), f32(nf), f32(nf)
        self.keys, self.values, self.hist, self.state = {}, {}, {}, {}
        for i in range(cfg.layers):
            if cfg.is_attention(i):
                self.keys[i] = f32(self.cap * nkv * D)
                self.values[i] = f32(self.cap * nkv * D)
            else:
                self.hist[i] = f32(2 * self.channels * cfg.conv_kernel)
                self.state[i] = f32(nv * D * D)
        self.rope_table = f32(self.cap * cfg.rope_dim)
        ctx.rope_table(cfg.rope_dim, cfg.rope_sections, cfg.rope_base, self.cap, self.rope_table)
        u32 = lambda n: torch.zeros(n, dtype=torch.int32, device=dev)  # noqa: E731
        self.pos, self.next_id = u32(1), u32(1)
        self.prompt, self.tokens = u32(self.cap), u32(self.max_new)
        self.key = torch.zeros(1, dtype=torch.int64, device=dev)
        self.stream = torch.cuda.Stream(device=dev)
        self.graph, self.graph_prompt = None, None
        self.timer = None  # list of (start, end) CUDA events around the program calls, when set
        self.deps_per_step = 2 * cfg.layers + 1
        ctx.set_flags(ctx.flags | FLAG_PDL | FLAG_BUILD_IN_KERNEL)

    # ---------------------------------------------------------------- weights
    def _put(self, name, qtype, dims, arr) -> None:
        host = self.torch.from_numpy(np.ascontiguousarray(arr))
        self.w[name] = (qtype, tuple(int(d) for d in dims), host.to(self.dev))

    def _load(self, t) -> None:
        cfg, plan, D = self.cfg, self.plan, self.cfg.state_size
        for name in ("token_embd.weight", "output_norm.weight"):
            self._put(name, *t[name])
        lm = "output.weight" if "output.weight" in t else "token_embd.weight"
        qt, dims, data = t[lm]
        rows = np.arange(plan.vocab_lo, plan.vocab_hi)
        self._put("lm_head", qt, (dims[0], rows.size), take_rows(data, qt, dims, rows))
        kw, fb = cfg.key_width, plan.ffn_blocks
        for i in range(cfg.layers):
            p = f"blk.{i}."
            for n in ("attn_norm.weight", "post_attention_norm.weight"):
                self._put(p + n, *t[p + n])
            if cfg.is_attention(i):
                for n, units, width in (("attn_q.weight", plan.q_heads, 2 * D), ("attn_k.weight", plan.kv_heads, D),
                                        ("attn_v.weight", plan.kv_heads, D)):
                    qt, dims, data = t[p + n]
                    rows = _ranges(units, width)
                    self._put(p + n, qt, (dims[0], rows.size), take_rows(data, qt, dims, rows))
                for n in ("attn_q_norm.weight", "attn_k_norm.weight"):
                    self._put(p + n, *t[p + n])
                out, blocks = "attn_output.weight", owned_blocks(cfg.q_width // BLOCK, plan.world, plan.rank)
            else:
                ch = np.concatenate([_ranges(plan.key_heads, D), kw + _ranges(plan.key_heads, D),
                                     2 * kw + _ranges(plan.value_heads, D)])
                qt, dims, data = t[p + "attn_qkv.weight"]
                self._put(p + "attn_qkv.weight", qt, (dims[0], ch.size), take_rows(data, qt, dims, ch))
                qt, dims, data = t[p + "ssm_conv1d.weight"]
                conv = data.view(np.float32).reshape(dims[1], dims[0])[ch]
                self._put(p + "ssm_conv1d.weight", qt, (dims[0], ch.size), conv.view(np.uint8).reshape(-1))
                for n, width in (("attn_gate.weight", D), ("ssm_beta.weight", 1), ("ssm_alpha.weight", 1)):
                    qt, dims, data = t[p + n]
                    rows = _ranges(plan.value_heads, width)
                    self._put(p + n, qt, (dims[0], rows.size), take_rows(data, qt, dims, rows))
                for n in ("ssm_dt.bias", "ssm_a"):
                    qt, dims, data = t[p + n]
                    vals = data.view(np.float32)[plan.value_heads]
                    self._put(p + n, qt, (vals.size,), vals.view(np.uint8))
                self._put(p + "ssm_norm.weight", *t[p + "ssm_norm.weight"])
                out, blocks = "ssm_out.weight", owned_blocks(cfg.value_width // BLOCK, plan.world, plan.rank)
            qt, dims, data = t[p + out]
            self._put(p + out, qt, (len(blocks) * BLOCK, dims[1]), take_blocks(data, qt, dims, blocks))
            for n in ("ffn_gate.weight", "ffn_up.weight"):
                qt, dims, data = t[p + n]
                rows = _ranges(fb, BLOCK)
                self._put(p + n, qt, (dims[0], rows.size), take_rows(data, qt, dims, rows))
            qt, dims, data = t[p + "ffn_down.weight"]
            for g in range(plan.ffn_segments):
                blocks = plan.ffn_segment_blocks(g)
                self._put(p + f"ffn_down.{g}", qt, (len(blocks) * BLOCK, dims[1]),
                          take_blocks(data, qt, dims, blocks))

    # ---------------------------------------------------------------- step
    def _vec(self, name):
        return self.w[name][2].view(self.torch.float32)

    def _op(self, name, x, y, **kw) -> dict:
        qtype, dims, w = self.w[name]
        return dict(qtype=qtype, rows=dims[1], cols=dims[0], w=w, x=x, y=y[:dims[1]], eps=self.cfg.eps, **kw)

    def _combine(self, partials, segments, norm, combined, wait) -> dict:
        return dict(xform=XFORM_COMBINE_RMS, x2=partials, segments=segments, norm=self._vec(norm),
                    combined=combined, wait=wait)

    def _input_projections(self, i: int, first: bool) -> list:
        """Block i's projections of this rank's heads from rms(hidden); after
        the first block hidden = resid + down(...), folded from every rank's
        ffn_down partials (qwen35_block.cpp:326-352, 441-463, 643-657)."""
        p = f"blk.{i}."
        names = ([("attn_q.weight", self.q_full), ("attn_k.weight", self.k), ("attn_v.weight", self.v)]
                 if self.cfg.is_attention(i) else
                 [("attn_qkv.weight", self.qkv), ("attn_gate.weight", self.z), ("ssm_beta.weight", self.beta),
                  ("ssm_alpha.weight", self.alpha)])
        ops = []
        for j, (n, y) in enumerate(names):
            if first:
                src = dict(xform=XFORM_RMS, norm=self._vec(p + "attn_norm.weight"))
                ops.append(self._op(p + n, self.hidden, y, **src))
            else:
                src = self._combine(self.part_down, self.plan.ffn_segments, p + "attn_norm.weight", self.hidden,
                                    2 if j == 0 else 3)
                ops.append(self._op(p + n, self.resid, y, **src))
        return ops

    def _block_tail(self, i: int) -> list:
        """Block i from its core's output to ffn_down's partial sums: the
        output projection over this rank's heads (partials of every row), then
        resid = hidden + out(x) folded from every rank, the gate / up rows of
        this rank's FFN columns from rms(resid), SwiGLU, and ffn_down over those
        columns, one partial per 16-block segment (qwen35_block.cpp:298-352)."""
        cfg, p, H, r = self.cfg, f"blk.{i}.", self.cfg.hidden, self.rank
        attn = cfg.is_attention(i)
        out, x = (p + "attn_output.weight", self.attn) if attn else (p + "ssm_out.weight", self.gated)
        ops = [self._op(out, x, self.part_out[r * H:(r + 1) * H], push=True, announce=True)]
        post = p + "post_attention_norm.weight"
        ops.append(self._op(p + "ffn_gate.weight", self.hidden, self.gate,
                            **self._combine(self.part_out, 1, post, self.resid, 2)))
        ops.append(self._op(p + "ffn_up.weight", self.hidden, self.up, swiglu_gate=self.gate, act=self.act,
                            **self._combine(self.part_out, 1, post, self.resid, 3)))
        G, off = self.plan.ffn_segments, 0
        for g in range(G):
            n = len(self.plan.ffn_segment_blocks(g)) * BLOCK
            y = self.part_down[(r * G + g) * H:(r * G + g + 1) * H]
            ops.append(self._op(p + f"ffn_down.{g}", self.act[off:off + n], y, push=True, wait=1 if g == 0 else 3,
                                announce=g == G - 1))
            off += n
        return ops

    def _lm_head(self) -> dict:
        """The final norm and this rank's vocabulary rows (qwen35_forward.cpp:446-466)."""
        lo, hi = self.plan.vocab_lo, self.plan.vocab_hi
        return self._op("lm_head", self.resid, self.logits[lo:hi], push=True, announce=True,
                        **self._combine(self.part_down, self.plan.ffn_segments, "output_norm.weight", self.hidden, 2))

    def _core(self, i: int, s) -> None:
        cfg, ctx, p, plan = self.cfg, self.ctx, f"blk.{i}.", self.plan
        D = cfg.head_dim
        if cfg.is_attention(i):
            nq, nkv = len(plan.q_heads), len(plan.kv_heads)
            ctx.attention_prep_at(self.q_full, self.k, self.v, self._vec(p + "attn_q_norm.weight"),
                                  self._vec(p + "attn_k_norm.weight"), cfg.eps, self.rope_table, cfg.rope_dim,
                                  nq, nkv, D, self.keys[i], self.values[i], self.cap, self.pos, self.qn, s)
            ctx.attention_core_at(self.qn, self.keys[i], self.values[i], self.cap, self.pos, nq, nkv, D, D,
                                  self.q_full[D:], 2 * D, self.scores, self.attn, s)
        else:
            ctx.gdn_core(self.qkv, self.z, self.beta, self.alpha, self._vec(p + "ssm_dt.bias"), self._vec(p + "ssm_a"),
                         self._vec(p + "ssm_conv1d.weight"), self.hist[i], self.state[i],
                         self._vec(p + "ssm_norm.weight"), len(plan.key_heads), len(plan.value_heads),
                         cfg.state_size, cfg.conv_kernel, cfg.eps, self.pos, self.gated, s)

    def _program(self, ops, first_dep: int, last: bool, s) -> None:
        if self.timer is not None:
            ev = (self.torch.cuda.Event(enable_timing=True), self.torch.cuda.Event(enable_timing=True))
            ev[0].record(self.stream)
        self.ctx.matvec_program_sharded(self.group, ops, first_dep, self.deps_per_step, end_of_step=last,
                                        tail_wait=last, stream=s)
        if self.timer is not None:
            ev[1].record(self.stream)
            self.timer.append((ev, sum(o["w"].numel() for o in ops)))

    def _enqueue_step(self, n_prompt: int, s) -> None:
        cfg, ctx, L = self.cfg, self.ctx, self.cfg.layers
        et, edims, emb = self.w["token_embd.weight"]
        ctx.gather_rows(et, edims[1], edims[0], emb, self.next_id, self.hidden, s)
        self._program(self._input_projections(0, True), 0, False, s)
        for i in range(L):
            self._core(i, s)
            last = i + 1 == L
            ops = self._block_tail(i) + ([self._lm_head()] if last else self._input_projections(i + 1, False))
            self._program(ops, 2 * i, last, s)
        ctx.argmax(self.logits, self.key, 0, s)
        ctx.token_commit(self.key, self.prompt, n_prompt, self.pos, self.next_id, self.tokens, self.max_new, s)

    # ---------------------------------------------------------------- control
    def reset(self) -> None:
        """Empty caches and states, position 0 (the cross-rank counters keep
        counting: every rank runs the same steps)."""
        with self.torch.cuda.stream(self.stream):
            for t in (*self.keys.values(), *self.values.values(), *self.hist.values(), *self.state.values()):
                t.zero_()
            self.pos.zero_()
            self.tokens.zero_()
        self.stream.synchronize()

    def capture(self, n_prompt: int) -> None:
        """One uncaptured warm-up step on every rank, then the step captured
        in a CUDA graph; the state is reset afterwards."""
        torch, s = self.torch, self.stream
        self.reset()
        self._enqueue_step(n_prompt, s.cuda_stream)
        s.synchronize()
        self.ctx.device_status()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            self._enqueue_step(n_prompt, s.cuda_stream)
        self.graph, self.graph_prompt = g, n_prompt
        self.reset()

    def step(self) -> None:
        with self.torch.cuda.stream(self.stream):
            self.graph.replay()

    def start(self, prompt) -> None:
        torch = self.torch
        prompt = np.ascontiguousarray(prompt, np.uint32)
        if prompt.size == 0 or prompt.size > self.cap:
            raise ValueError("prompt must hold 1 .. capacity tokens")
        if self.graph is None or self.graph_prompt != prompt.size:
            self.capture(int(prompt.size))
        self.reset()
        with torch.cuda.stream(self.stream):
            self.prompt[:prompt.size].copy_(torch.from_numpy(prompt.view(np.int32)).to(self.dev))
            self.next_id.fill_(int(prompt[0]))
        self.stream.synchronize()

    def generate(self, prompt, n_new: int) -> np.ndarray:
        """Fresh greedy generation (every rank returns the same tokens)."""
        if not 1 <= n_new <= self.max_new:
            raise ValueError(f"n_new must be in [1, {self.max_new}]")
        self.start(prompt)
        with self.torch.cuda.stream(self.stream):
            for _ in range(len(prompt) + n_new - 1):
                self.graph.replay()
        self.stream.synchronize()
        self.ctx.device_status()
        return self.tokens[:n_new].cpu().numpy().view(np.uint32).copy()

    def forward(self, token: int) -> np.ndarray:
        """One step on `token` at the current position: the whole logits."""
        if self.graph is None:
            self.capture(1)
        with self.torch.cuda.stream(self.stream):
            self.next_id.fill_(int(token))
            self.graph.replay()
        self.stream.synchronize()
        self.ctx.device_status()
        return self.logits.cpu().numpy().copy()

    def profile_projections(self) -> tuple:
        """One uncaptured step with CUDA events around every program call:
        (this rank's weight bytes they stream, their summed milliseconds, the
        step's milliseconds).  The state is reset afterwards."""
        torch = self.torch
        self.timer = []
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(self.stream)
        self._enqueue_step(self.graph_prompt or 1, self.stream.cuda_stream)
        b.record(self.stream)
        self.stream.synchronize()
        timer, self.timer = self.timer, None
        self.reset()
        return (sum(n for _, n in timer), sum(e[0].elapsed_time(e[1]) for e, _ in timer), a.elapsed_time(b))

    def launches_per_step(self) -> int:
        """Kernels one step launches (counted on an uncaptured step)."""
        before = self.ctx.launch_count()
        self._enqueue_step(self.graph_prompt or 1, self.stream.cuda_stream)
        self.stream.synchronize()
        n = self.ctx.launch_count() - before
        self.reset()
        return n

    def weight_bytes(self) -> int:
        """Bytes of the matrices one step streams on this rank (projections,
        the LM-head rows; not the embedding table, of which it reads one row)."""
        return sum(w.numel() for n, (qt, dims, w) in self.w.items()
                   if len(dims) == 2 and qt != TYPE_F32 and n != "token_embd.weight")

    def close(self) -> None:
        """Release the graph and the peer group (before the process group goes)."""
        self.graph = None
        if self.group is not None:
            self.stream.synchronize()
            self.group.close()
            self.group = None
