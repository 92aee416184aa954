"""Batched greedy decoding: up to 16 sequences of the Qwen3.5 hybrid model in
lockstep on one B200.

Oracle decodes one sequence per call of execute_qwen35_reference_token
(src/runtime/qwen35_forward.cpp:400-470); serving many requests repeats that
loop per request, and every token of every request streams every weight byte
once.  Here B sequences (same prompt length, so one shared position) take each
step together, and every projection reads its weights ONCE for all of them:

* activations are stacked [B][width]; each projection input is quantized once
  into a batch image (``Context.batch_quantize``) that every matrix reading it
  shares, and each matrix is one ``Context.batch_matvec`` (int8 tensor-core
  MMAs, bit-identical per sequence to the single-vector Q8_K kernels);
* RMSNorm, with the residual add before it, is fused into the quantization
  of the projection input it feeds (one launch); SwiGLU is a row-wise kernel;
* attention runs the sequences as B x heads query heads over a KV cache laid
  out [token][sequence][kv_head][dim] (a GQA group never crosses a sequence),
  with the batch-1 decoder's fused prep / core kernels unchanged;
* the recurrent block core (``gdn_core_seqs``) runs one CTA row per sequence
  on that sequence's history and state;
* sampling is a per-row argmax and one commit kernel that feeds each sequence
  its next prompt token or its sampled token, then advances the position.

Every operation is per sequence, so sequence b's logits and tokens are those
of the same decoder run with B = 1 on sequence b alone, bit for bit (tested),
and its greedy tokens are Oracle's for that prompt (tested against the
reference's decode loop).  The step is captured in a CUDA graph after one
warm-up step and replayed per token, as in ``Qwen35Decoder``.
"""
from __future__ import annotations

import numpy as np

from . import FLAG_PDL, TYPE_F32, TYPE_Q4_K, TYPE_Q6_K, Context
from .qwen35 import Qwen35Config

MAX_BATCH = 16


class BatchDecoder:
    """B (1..16) sequences of one resident Q4_K / Q6_K model, decoded together.

    tensors: [(name, ggml type, gguf dims, uint8 bytes)] as for
    ``Qwen35Decoder``; projections must be q4_K or q6_K (the Q8_K contract)."""

    def __init__(self, ctx: Context, cfg: Qwen35Config, tensors, batch: int, capacity: int | None = None,
                 max_new: int = 4096, device: int = 0):
        import torch

        if not 1 <= batch <= MAX_BATCH:
            raise ValueError(f"batch must be in [1, {MAX_BATCH}]")
        self.torch, self.ctx, self.cfg, self.B = torch, ctx, cfg, int(batch)
        self.dev = dev = torch.device("cuda", device)
        self.cap = int(capacity or cfg.context)
        self.max_new = int(max_new)
        self.w = {}
        for name, qtype, dims, data in tensors:
            arr = np.ascontiguousarray(data).view(np.uint8)
            host = torch.from_numpy(arr if arr.flags.writeable else arr.copy())
            self.w[name] = (int(qtype), tuple(dims), host.to(dev))
            if len(dims) == 2 and qtype not in (TYPE_F32, TYPE_Q4_K, TYPE_Q6_K) and name != "token_embd.weight":
                raise ValueError(f"{name}: batched decoding runs Q4_K / Q6_K matrices only")
        B, H, F = self.B, cfg.hidden, cfg.ffn
        f32 = lambda n: torch.zeros(n, dtype=torch.float32, device=dev)  # noqa: E731
        self.hidden, self.resid, self.branch, self.ffn_out = (f32(B * H) for _ in range(4))
        self.ffn_gate, self.ffn_up, self.ffn_act = f32(B * F), f32(B * F), f32(B * F)
        widest = max(H, F, cfg.q_width, cfg.value_width)
        self.image = torch.zeros(Context.batch_image_bytes(widest), dtype=torch.uint8, device=dev)
        # recurrent blocks
        self.qkv, self.z = f32(B * cfg.conv_channels), f32(B * cfg.value_width)
        self.beta, self.alpha = f32(B * cfg.value_heads), f32(B * cfg.value_heads)
        self.gated = f32(B * cfg.value_width)
        # attention blocks: the sequences as B x heads heads
        self.q_full, self.k, self.v = f32(B * 2 * cfg.q_width), f32(B * cfg.kv_width), f32(B * cfg.kv_width)
        self.qn, self.attn = f32(B * cfg.q_width), f32(B * cfg.q_width)
        self.scores = f32(B * cfg.heads * self.cap)
        self.keys, self.values, self.hist, self.state = {}, {}, {}, {}
        for i in range(cfg.layers):
            if cfg.is_attention(i):
                self.keys[i] = f32(self.cap * B * cfg.kv_width)
                self.values[i] = f32(self.cap * B * cfg.kv_width)
            else:
                self.hist[i] = f32(B * 2 * cfg.conv_channels * cfg.conv_kernel)
                self.state[i] = f32(B * cfg.value_heads * cfg.state_size * cfg.state_size)
        self.rope_table = f32(self.cap * cfg.rope_dim)
        ctx.rope_table(cfg.rope_dim, cfg.rope_sections, cfg.rope_base, self.cap, self.rope_table)
        self.logits = f32(B * cfg.vocab)
        u32 = lambda n: torch.zeros(n, dtype=torch.int32, device=dev)  # noqa: E731
        self.pos, self.next_id = u32(1), u32(B)
        self.prompt, self.tokens = u32(B * self.cap), u32(B * self.max_new)
        self.am_keys = torch.zeros(B, dtype=torch.int64, device=dev)
        self.stream = torch.cuda.Stream(device=dev)
        self.graph, self.graph_prompt = None, None
        self.timer = None  # list of (start, end) CUDA events around the matvecs, when set
        ctx.set_flags(ctx.flags | FLAG_PDL)

    # ---------------------------------------------------------------- pieces
    def _vec(self, name):
        return self.w[name][2].view(self.torch.float32)

    def _quantize(self, x, cols, s) -> None:
        self.ctx.batch_quantize(x, cols, self.B, self.image, s)

    def _mv(self, name, y, s) -> None:
        """y[b] = W x_b for every sequence, x the last quantized input."""
        qtype, dims, w = self.w[name]
        if self.timer is not None:
            ev = (self.torch.cuda.Event(enable_timing=True), self.torch.cuda.Event(enable_timing=True))
            ev[0].record(self.stream)
        self.ctx.batch_matvec(qtype, dims[1], dims[0], w, self.image, self.B, y[:self.B * dims[1]], s)
        if self.timer is not None:
            ev[1].record(self.stream)
            self.timer.append((ev, w.numel()))

    def _recurrent(self, i: int, s) -> None:
        cfg, p = self.cfg, f"blk.{i}."
        self._mv(p + "attn_qkv.weight", self.qkv, s)
        self._mv(p + "attn_gate.weight", self.z, s)
        self._mv(p + "ssm_beta.weight", self.beta, s)
        self._mv(p + "ssm_alpha.weight", self.alpha, s)
        self.ctx.gdn_core_seqs(self.qkv, self.z, self.beta, self.alpha, self._vec(p + "ssm_dt.bias"),
                               self._vec(p + "ssm_a"), self._vec(p + "ssm_conv1d.weight"), self.hist[i],
                               self.state[i], self._vec(p + "ssm_norm.weight"), cfg.key_heads, cfg.value_heads,
                               cfg.state_size, cfg.conv_kernel, cfg.eps, self.pos, self.B, self.gated, s)
        self._quantize(self.gated, cfg.value_width, s)
        self._mv(p + "ssm_out.weight", self.branch, s)

    def _attention(self, i: int, s) -> None:
        cfg, ctx, p, B = self.cfg, self.ctx, f"blk.{i}.", self.B
        D = cfg.head_dim
        self._mv(p + "attn_q.weight", self.q_full, s)
        self._mv(p + "attn_k.weight", self.k, s)
        self._mv(p + "attn_v.weight", self.v, s)
        ctx.attention_prep_at(self.q_full, self.k, self.v, self._vec(p + "attn_q_norm.weight"),
                              self._vec(p + "attn_k_norm.weight"), cfg.eps, self.rope_table, cfg.rope_dim,
                              B * cfg.heads, B * cfg.kv_heads, D, self.keys[i], self.values[i], self.cap, self.pos,
                              self.qn, s)
        ctx.attention_core_at(self.qn, self.keys[i], self.values[i], self.cap, self.pos, B * cfg.heads,
                              B * cfg.kv_heads, D, D, self.q_full[D:], 2 * D, self.scores, self.attn, s)
        self._quantize(self.attn, cfg.q_width, s)
        self._mv(p + "attn_output.weight", self.branch, s)

    def _enqueue_step(self, n_prompt: int, s) -> None:
        cfg, ctx, B = self.cfg, self.ctx, self.B
        H, F = cfg.hidden, cfg.ffn
        et, edims, emb = self.w["token_embd.weight"]
        ctx.gather_rows(et, edims[1], edims[0], emb, self.next_id, self.hidden, s)
        # the residual adds and norms are fused into the quantization of the
        # projection input they feed: hidden = resid + ffn_out (the previous
        # block's end) with this block's input norm, resid = hidden + branch
        # with the post-attention norm (finish_block, qwen35_block.cpp:326-352)
        ctx.batch_norm_quantize(self.hidden, None, None, self._vec("blk.0.attn_norm.weight"), cfg.eps, H, B,
                                self.image, s)
        for i in range(cfg.layers):
            p = f"blk.{i}."
            if cfg.is_attention(i):
                self._attention(i, s)
            else:
                self._recurrent(i, s)
            ctx.batch_norm_quantize(self.hidden, self.branch, self.resid, self._vec(p + "post_attention_norm.weight"),
                                    cfg.eps, H, B, self.image, s)
            self._mv(p + "ffn_gate.weight", self.ffn_gate, s)
            self._mv(p + "ffn_up.weight", self.ffn_up, s)
            ctx.swiglu(self.ffn_gate, self.ffn_up, B * F, self.ffn_act, s)
            self._quantize(self.ffn_act, F, s)
            self._mv(p + "ffn_down.weight", self.ffn_out, s)
            nxt = f"blk.{i + 1}.attn_norm.weight" if i + 1 < cfg.layers else "output_norm.weight"
            ctx.batch_norm_quantize(self.resid, self.ffn_out, self.hidden, self._vec(nxt), cfg.eps, H, B, self.image, s)
        self._mv("output.weight" if "output.weight" in self.w else "token_embd.weight", self.logits, s)
        ctx.argmax_rows(self.logits, B, cfg.vocab, self.am_keys, s)
        ctx.token_commit_rows(self.am_keys, B, self.prompt, n_prompt, self.pos, self.next_id, self.tokens,
                              self.max_new, s)

    # ---------------------------------------------------------------- control
    def reset(self) -> None:
        """Empty every sequence's caches and states, position 0."""
        with self.torch.cuda.stream(self.stream):
            for t in (*self.keys.values(), *self.values.values(), *self.hist.values(), *self.state.values()):
                t.zero_()
            self.pos.zero_()
            self.tokens.zero_()
            self.am_keys.zero_()
        self.stream.synchronize()

    def capture(self, n_prompt: int) -> None:
        """Capture the step in a CUDA graph after one uncaptured warm-up step
        (which sizes the context's scratch); the state is reset afterwards."""
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

    def start(self, prompts) -> None:
        """Reset and load one prompt per sequence ([B][n], one length)."""
        torch = self.torch
        prompts = np.ascontiguousarray(prompts, np.uint32)
        if prompts.ndim != 2 or prompts.shape[0] != self.B:
            raise ValueError(f"prompts must be a [{self.B}][n] array")
        n = prompts.shape[1]
        if n == 0 or n > self.cap:
            raise ValueError("prompts must hold 1 .. capacity tokens")
        if self.graph is None or self.graph_prompt != n:
            self.capture(n)
        self.reset()
        with torch.cuda.stream(self.stream):
            self.prompt[:self.B * n].copy_(torch.from_numpy(prompts.reshape(-1).view(np.int32)).to(self.dev))
            self.next_id.copy_(torch.from_numpy(prompts[:, 0].copy().view(np.int32)).to(self.dev))
        self.stream.synchronize()

    def step(self) -> None:
        """Replay one captured step on the decoder's stream (asynchronous)."""
        with self.torch.cuda.stream(self.stream):
            self.graph.replay()

    def generate(self, prompts, n_new: int) -> np.ndarray:
        """Fresh greedy generation for every sequence: [B][n_new] tokens."""
        if not 1 <= n_new <= self.max_new:
            raise ValueError(f"n_new must be in [1, {self.max_new}]")
        prompts = np.ascontiguousarray(prompts, np.uint32)
        self.start(prompts)
        with self.torch.cuda.stream(self.stream):
            for _ in range(prompts.shape[1] + n_new - 1):
                self.graph.replay()
        self.stream.synchronize()
        self.ctx.device_status()
        toks = self.tokens.view(self.B, self.max_new)[:, :n_new]
        return toks.cpu().numpy().view(np.uint32).copy()

    def forward(self, tokens) -> np.ndarray:
        """One step on tokens[b] for every sequence at the current position:
        the [B][vocab] logits."""
        if self.graph is None:
            self.capture(1)
        ids = np.ascontiguousarray(tokens, np.uint32).reshape(self.B)
        with self.torch.cuda.stream(self.stream):
            self.next_id.copy_(self.torch.from_numpy(ids.view(np.int32)).to(self.dev))
            self.graph.replay()
        self.stream.synchronize()
        self.ctx.device_status()
        return self.logits.view(self.B, self.cfg.vocab).cpu().numpy().copy()

    def profile_projections(self) -> tuple:
        """One uncaptured step with CUDA events around every batched matvec:
        (weight bytes they stream, their summed milliseconds, the step's
        milliseconds).  The state is reset afterwards."""
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
        """Kernels one step launches (counted by the context on an uncaptured step)."""
        before = self.ctx.launch_count()
        self._enqueue_step(self.graph_prompt or 1, self.stream.cuda_stream)
        self.stream.synchronize()
        n = self.ctx.launch_count() - before
        self.reset()
        return n

    def close(self) -> None:
        self.graph = None
