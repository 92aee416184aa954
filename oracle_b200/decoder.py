"""Greedy decoding of the Qwen3.5 hybrid model on one B200.

The per-token step is Oracle's execute_qwen35_reference_token
(src/runtime/qwen35_forward.cpp:400-470) with its blocks
(src/runtime/qwen35_block.cpp: recurrent 407-604, attention 606-760, MLP and
residual 300-352) laid out as a sequence of this library's kernels on one
stream, captured once in a CUDA graph and replayed for every token:

* every weight stays resident in HBM in its GGML bytes; the projections of a
  block that read the same input run as ONE matvec program (Q8_K contract:
  ``qkv/z/beta/alpha``, ``q/k/v``, ``gate/up``), or one Oracle-f32-contract
  matvec each (``contract="f32"``);
* the KV caches (f32, [token][kv_head][dim]), convolution histories and
  recurrent states live on the device; the token position is a device counter
  read by RoPE (a cos/sin table of every position) and attention, so the
  graph is position-independent;
* sampling stays on the device: argmax of the logits into a 64-bit key,
  then ``token_commit`` picks the next input id (the next prompt token while
  the prompt lasts, else the sampled token, which it also records) and
  advances the position.  A whole generation is graph replays with no host
  round trip; the host reads the tokens once at the end.
"""
from __future__ import annotations

import numpy as np

from . import CONTRACT_F32, FLAG_BUILD_IN_KERNEL, FLAG_PDL, XFORM_RMS, XFORM_SWIGLU, Context, TYPE_F32, TYPE_Q4_K, TYPE_Q6_K
from .qwen35 import Qwen35Config


def tensors_from_gguf(path: str) -> tuple:
    """(Qwen35Config, [(name, ggml type, gguf dims, uint8 bytes)]) of a
    Qwen3.5 GGUF file, read with gguf-py's memory-mapped reader; metadata keys
    as Oracle's load_qwen35_manifest reads them (qwen35_manifest.cpp:151-206)."""
    import gguf

    r = gguf.GGUFReader(path)

    def val(key):
        f = r.fields[key]
        return f.parts[f.data[0]].tolist()[0] if len(f.data) == 1 else [f.parts[i].tolist()[0] for i in f.data]

    cfg = Qwen35Config(
        hidden=val("qwen35.embedding_length"), ffn=val("qwen35.feed_forward_length"),
        layers=val("qwen35.block_count"), heads=val("qwen35.attention.head_count"),
        kv_heads=val("qwen35.attention.head_count_kv"), head_dim=val("qwen35.attention.key_length"),
        rope_dim=val("qwen35.rope.dimension_count"), rope_sections=tuple(val("qwen35.rope.dimension_sections")),
        rope_base=float(val("qwen35.rope.freq_base")), conv_kernel=val("qwen35.ssm.conv_kernel"),
        state_size=val("qwen35.ssm.state_size"), key_heads=val("qwen35.ssm.group_count"),
        value_heads=val("qwen35.ssm.time_step_rank"), vocab=len(r.fields["tokenizer.ggml.tokens"].data),
        eps=float(val("qwen35.attention.layer_norm_rms_epsilon")),
        interval=val("qwen35.full_attention_interval"), context=val("qwen35.context_length"))
    tensors = []
    for t in r.tensors:
        dims = tuple(int(d) for d in t.shape)
        tensors.append((t.name, int(t.tensor_type), dims, np.asarray(t.data).view(np.uint8).reshape(-1)))
    return cfg, tensors


class Qwen35Decoder:
    """Resident weights, device state and the captured decode step of one model.

    tensors: [(name, ggml type, gguf dims, uint8 bytes)] as produced by
    ``qwen35.synthetic_model`` or ``tensors_from_gguf``.  contract "q8k"
    (GGML's Q8_K activations; Q4_K / Q6_K matrices) or "f32" (Oracle's own
    f32 contract; any storage type the reference admits)."""

    def __init__(self, ctx: Context, cfg: Qwen35Config, tensors, contract: str = "q8k",
                 capacity: int | None = None, max_new: int = 4096, device: int = 0, fused: bool = True,
                 rank: int = 0, world: int = 1, exchange=None, build_in_kernel: bool = True):
        import torch

        if contract not in ("q8k", "f32"):
            raise ValueError("contract must be 'q8k' or 'f32'")
        if world > 1 and (contract != "q8k" or not fused or exchange is None):
            raise ValueError("several GPUs need the fused Q8_K step and an `exchange` of peer handles")
        self.torch = torch
        self.ctx, self.cfg, self.contract = ctx, cfg, contract
        self.rank, self.world = rank, world
        # fused (Q8_K contract only): one matvec program per block boundary
        # (output projection + MLP + the next block's input projections, norms,
        # SwiGLU and residual adds applied inside) and one kernel per block core
        self.fused = fused and contract == "q8k"
        self.dev = torch.device("cuda", device)
        self.cap = int(capacity or cfg.context)
        self.max_new = int(max_new)
        dev = self.dev
        # Several GPUs: every projection's rows are split evenly over the ranks
        # (each rank uploads only its rows); the outputs of every projection
        # live in a peer group's gather buffer, which the programs fill on every
        # rank over NVLink; the block cores, the embedding and the sampling run
        # on every rank on the whole vectors (they are small), so every rank
        # holds the same state and produces the same tokens as one GPU.
        self.w, self.shard = {}, {}
        for name, qtype, dims, data in tensors:
            arr = np.ascontiguousarray(data).view(np.uint8)
            if world > 1 and len(dims) == 2 and name not in ("token_embd.weight",) and qtype != TYPE_F32:
                rows = dims[1]
                rb = arr.size // rows
                lo, hi = rank * rows // world, (rank + 1) * rows // world
                arr = arr[lo * rb:hi * rb]
                self.shard[name] = (lo, hi - lo)
            host = torch.from_numpy(arr if arr.flags.writeable else arr.copy())
            self.w[name] = (int(qtype), tuple(dims), host.to(dev))
            if contract == "q8k" and len(dims) == 2 and qtype not in (TYPE_F32, TYPE_Q4_K, TYPE_Q6_K) \
                    and name != "token_embd.weight":
                raise ValueError(f"{name}: the Q8_K contract runs Q4_K / Q6_K matrices only")
        H, F = cfg.hidden, cfg.ffn
        f32 = lambda n: torch.zeros(n, dtype=torch.float32, device=dev)  # noqa: E731
        gathered = dict(hidden=H, resid=H, ffn_gate=F, ffn_up=F, ffn_act=F, qkv=cfg.conv_channels,
                        z=cfg.value_width, beta=cfg.value_heads, alpha=cfg.value_heads, q_full=2 * cfg.q_width,
                        k=cfg.kv_width, v=cfg.kv_width, logits=cfg.vocab)
        self.group = None
        if world > 1:
            from . import PeerGroup
            sizes = {k: (n + 3) // 4 * 4 for k, n in gathered.items()}  # 16-byte aligned vectors
            self.group = PeerGroup(ctx, rank, world, sum(sizes.values()) * 4)
            self.group.connect(exchange(self.group.handle))
            data, off = self.group.tensor(), 0
            for k, n in gathered.items():
                setattr(self, k, data[off:off + n])
                off += sizes[k]
        else:
            for k, n in gathered.items():
                setattr(self, k, f32(n))
        self.normed, self.branch, self.ffn_out = f32(H), f32(H), f32(H)
        # recurrent blocks
        self.conv_out = f32(cfg.conv_channels)
        self.beta_s, self.log_decay = f32(cfg.value_heads), f32(cfg.value_heads)
        self.rec_out, self.gated = f32(cfg.value_width), f32(cfg.value_width)
        # attention blocks
        self.q, self.gate = f32(cfg.q_width), f32(cfg.q_width)
        self.qn, self.kn = f32(cfg.q_width), f32(cfg.kv_width)
        self.attn, self.scores = f32(cfg.q_width), f32(cfg.heads * self.cap)
        self.keys, self.values, self.hist, self.state = {}, {}, {}, {}
        for i in range(cfg.layers):
            if cfg.is_attention(i):
                self.keys[i] = f32(self.cap * cfg.kv_width)
                self.values[i] = f32(self.cap * cfg.kv_width)
            else:
                # the fused core double-buffers the history by position parity
                self.hist[i] = f32((2 if self.fused else 1) * cfg.conv_channels * cfg.conv_kernel)
                self.state[i] = f32(cfg.value_heads * cfg.state_size * cfg.state_size)
        self.rope_table = f32(self.cap * cfg.rope_dim)
        ctx.rope_table(cfg.rope_dim, cfg.rope_sections, cfg.rope_base, self.cap, self.rope_table)
        u32 = lambda n: torch.zeros(n, dtype=torch.int32, device=dev)  # noqa: E731
        self.pos, self.next_id = u32(1), u32(1)
        self.prompt, self.tokens = u32(self.cap), u32(self.max_new)
        self.key = torch.zeros(1, dtype=torch.int64, device=dev)
        self.stream = torch.cuda.Stream(device=dev)
        self.graph, self.graph_prompt = None, None
        # programmatic dependent launch: each kernel of the step launches while
        # its predecessor drains (programs start streaming weights early)
        if self.fused:
            ctx.set_flags(ctx.flags | FLAG_PDL | (FLAG_BUILD_IN_KERNEL if build_in_kernel else 0))
        self.timer = None  # list of (start, end) CUDA events around projections, when set

    # ---------------------------------------------------------------- pieces
    def _t(self, name):
        return self.w[name][2]

    def _vec(self, name):
        return self.w[name][2].view(self.torch.float32)

    def _project(self, ops, s) -> None:
        """ops: [(weight name, x, y)] that read inputs produced before the call."""
        if self.timer is not None:
            ev = (self.torch.cuda.Event(enable_timing=True), self.torch.cuda.Event(enable_timing=True))
            ev[0].record(self.stream)
        if self.contract == "q8k":
            prog = []
            for name, x, y in ops:
                qtype, dims, w = self.w[name]
                prog.append((qtype, dims[1], dims[0], w, x, y, False))
            self.ctx.matvec_program(prog, s)
        else:
            for name, x, y in ops:
                qtype, dims, w = self.w[name]
                self.ctx.storage_matvec(CONTRACT_F32, qtype, dims[1], dims[0], w, x, y, s)
        if self.timer is not None:
            ev[1].record(self.stream)
            self.timer.append((ev, sum(self.w[name][2].numel() for name, _, _ in ops)))

    def _recurrent(self, i: int, s) -> None:
        cfg, ctx, p = self.cfg, self.ctx, f"blk.{i}."
        self._project([(p + "attn_qkv.weight", self.normed, self.qkv), (p + "attn_gate.weight", self.normed, self.z),
                       (p + "ssm_beta.weight", self.normed, self.beta),
                       (p + "ssm_alpha.weight", self.normed, self.alpha)], s)
        ctx.gdn_gates(self.beta, self.alpha, self._vec(p + "ssm_dt.bias"), self._vec(p + "ssm_a"), cfg.value_heads,
                      self.beta_s, self.log_decay, s)
        ctx.conv_step(self.qkv, self._vec(p + "ssm_conv1d.weight"), self.hist[i], cfg.conv_channels,
                      cfg.conv_kernel, True, self.conv_out, s)
        kw = cfg.key_width
        ctx.gated_delta_step(self.conv_out[:kw], self.conv_out[kw:2 * kw], self.conv_out[2 * kw:], self.beta_s,
                             self.log_decay, self.state[i], cfg.value_heads, cfg.state_size, cfg.state_size, cfg.eps,
                             self.rec_out, s, qk_heads=cfg.key_heads)
        ctx.rms_norm_rows(self.rec_out, self._vec(p + "ssm_norm.weight"), cfg.value_heads, cfg.state_size, cfg.eps,
                          self.gated, s)
        ctx.mul_silu(self.gated, self.z, cfg.value_width, s)
        self._project([(p + "ssm_out.weight", self.gated, self.branch)], s)

    def _attention(self, i: int, s) -> None:
        cfg, ctx, p = self.cfg, self.ctx, f"blk.{i}."
        self._project([(p + "attn_q.weight", self.normed, self.q_full), (p + "attn_k.weight", self.normed, self.k),
                       (p + "attn_v.weight", self.normed, self.v)], s)
        ctx.split_query_gate(self.q_full, cfg.heads, cfg.head_dim, self.q, self.gate, s)
        ctx.rms_norm_rows(self.q, self._vec(p + "attn_q_norm.weight"), cfg.heads, cfg.head_dim, cfg.eps, self.qn, s)
        ctx.rms_norm_rows(self.k, self._vec(p + "attn_k_norm.weight"), cfg.kv_heads, cfg.head_dim, cfg.eps, self.kn,
                          s)
        ctx.rope_at(self.qn, cfg.heads, cfg.head_dim, cfg.rope_dim, self.rope_table, self.cap, self.pos, s)
        ctx.rope_at(self.kn, cfg.kv_heads, cfg.head_dim, cfg.rope_dim, self.rope_table, self.cap, self.pos, s)
        ctx.attention_step_at(self.qn, self.kn, self.v, self.keys[i], self.values[i], self.cap, self.pos, cfg.heads,
                              cfg.kv_heads, cfg.head_dim, cfg.head_dim, self.scores, self.attn, s)
        ctx.gate_sigmoid_mul(self.attn, self.gate, cfg.q_width, s)
        self._project([(p + "attn_output.weight", self.attn, self.branch)], s)

    # ---------------------------------------------------------------- fused step
    def _mv(self, name, x, y, after=False, xform=0, x2=None, norm=None, residual=None, act=None) -> dict:
        """One program op; on several GPUs, this rank's rows of it."""
        qtype, dims, w = self.w[name]
        lo, n = self.shard.get(name, (0, dims[1]))
        return dict(qtype=qtype, rows=n, cols=dims[0], w=w, x=x, y=y[lo:lo + n], after=after, xform=xform,
                    eps=self.cfg.eps, x2=x2, norm=norm, residual=None if residual is None else residual[lo:lo + n],
                    act=act)

    def _input_projections(self, i: int, after: bool) -> list:
        """Block i's projections of rms_norm(hidden) (qwen35_block.cpp:441-463, 643-657)."""
        p = f"blk.{i}."
        kw = dict(after=after, xform=XFORM_RMS, norm=self._vec(p + "attn_norm.weight"))
        if self.cfg.is_attention(i):
            return [self._mv(p + "attn_q.weight", self.hidden, self.q_full, **kw),
                    self._mv(p + "attn_k.weight", self.hidden, self.k, **kw),
                    self._mv(p + "attn_v.weight", self.hidden, self.v, **kw)]
        return [self._mv(p + "attn_qkv.weight", self.hidden, self.qkv, **kw),
                self._mv(p + "attn_gate.weight", self.hidden, self.z, **kw),
                self._mv(p + "ssm_beta.weight", self.hidden, self.beta, **kw),
                self._mv(p + "ssm_alpha.weight", self.hidden, self.alpha, **kw)]

    def _block_tail(self, i: int) -> list:
        """Block i's output projection and MLP with finish_block's adds and norm
        (qwen35_block.cpp:298-352): resid = hidden + out(x); hidden = resid +
        down(silu(gate(rms(resid))) * up(rms(resid)))."""
        p = f"blk.{i}."
        attn = self.cfg.is_attention(i)
        out, x = (p + "attn_output.weight", self.attn) if attn else (p + "ssm_out.weight", self.gated)
        post = dict(after=True, xform=XFORM_RMS, norm=self._vec(p + "post_attention_norm.weight"))
        return [self._mv(out, x, self.resid, residual=self.hidden),
                self._mv(p + "ffn_gate.weight", self.resid, self.ffn_gate, **post),
                self._mv(p + "ffn_up.weight", self.resid, self.ffn_up, **post),
                self._mv(p + "ffn_down.weight", self.ffn_gate, self.hidden, after=True, xform=XFORM_SWIGLU,
                         x2=self.ffn_up, residual=self.resid, act=self.ffn_act)]

    def _core(self, i: int, s) -> None:
        cfg, ctx, p = self.cfg, self.ctx, f"blk.{i}."
        D = cfg.head_dim
        if cfg.is_attention(i):
            ctx.attention_prep_at(self.q_full, self.k, self.v, self._vec(p + "attn_q_norm.weight"),
                                  self._vec(p + "attn_k_norm.weight"), cfg.eps, self.rope_table, cfg.rope_dim,
                                  cfg.heads, cfg.kv_heads, D, self.keys[i], self.values[i], self.cap, self.pos,
                                  self.qn, s)
            ctx.attention_core_at(self.qn, self.keys[i], self.values[i], self.cap, self.pos, cfg.heads, cfg.kv_heads,
                                  D, D, self.q_full[D:], 2 * D, self.scores, self.attn, s)
        else:
            ctx.gdn_core(self.qkv, self.z, self.beta, self.alpha, self._vec(p + "ssm_dt.bias"),
                         self._vec(p + "ssm_a"), self._vec(p + "ssm_conv1d.weight"), self.hist[i], self.state[i],
                         self._vec(p + "ssm_norm.weight"), cfg.key_heads, cfg.value_heads, cfg.state_size,
                         cfg.conv_kernel, cfg.eps, self.pos, self.gated, s)

    def _program(self, ops, s) -> None:
        if self.timer is not None:
            ev = (self.torch.cuda.Event(enable_timing=True), self.torch.cuda.Event(enable_timing=True))
            ev[0].record(self.stream)
        if self.group is not None:
            self.ctx.matvec_program_ex_allgather(self.group, ops, s)
        else:
            self.ctx.matvec_program_ex(ops, s)
        if self.timer is not None:
            ev[1].record(self.stream)
            self.timer.append((ev, sum(o["w"].numel() for o in ops)))

    def _enqueue_fused_step(self, n_prompt: int, s) -> None:
        cfg, ctx = self.cfg, self.ctx
        et, edims, emb = self.w["token_embd.weight"]
        ctx.gather_rows(et, edims[1], edims[0], emb, self.next_id, self.hidden, s)
        self._program(self._input_projections(0, after=False), s)
        out = "output.weight" if "output.weight" in self.w else "token_embd.weight"
        for i in range(cfg.layers):
            self._core(i, s)
            ops = self._block_tail(i)
            if i + 1 < cfg.layers:
                ops += self._input_projections(i + 1, after=True)
            else:  # the final norm and the LM head (qwen35_forward.cpp:446-466)
                ops.append(self._mv(out, self.hidden, self.logits, after=True, xform=XFORM_RMS,
                                    norm=self._vec("output_norm.weight")))
            self._program(ops, s)
        ctx.argmax(self.logits, self.key, 0, s)
        ctx.token_commit(self.key, self.prompt, n_prompt, self.pos, self.next_id, self.tokens, self.max_new, s)

    def _enqueue_step(self, n_prompt: int, s) -> None:
        if self.fused:
            self._enqueue_fused_step(n_prompt, s)
            return
        cfg, ctx = self.cfg, self.ctx
        H = cfg.hidden
        et, edims, emb = self.w["token_embd.weight"]
        ctx.gather_rows(et, edims[1], edims[0], emb, self.next_id, self.hidden, s)
        for i in range(cfg.layers):
            p = f"blk.{i}."
            ctx.rms_norm_rows(self.hidden, self._vec(p + "attn_norm.weight"), 1, H, cfg.eps, self.normed, s)
            if cfg.is_attention(i):
                self._attention(i, s)
            else:
                self._recurrent(i, s)
            # finish_block (qwen35_block.cpp:326-352)
            ctx.add(self.hidden, self.branch, H, self.resid, s)
            ctx.rms_norm_rows(self.resid, self._vec(p + "post_attention_norm.weight"), 1, H, cfg.eps, self.normed, s)
            self._project([(p + "ffn_gate.weight", self.normed, self.ffn_gate),
                           (p + "ffn_up.weight", self.normed, self.ffn_up)], s)
            ctx.swiglu(self.ffn_gate, self.ffn_up, cfg.ffn, self.ffn_act, s)
            self._project([(p + "ffn_down.weight", self.ffn_act, self.ffn_out)], s)
            ctx.add(self.resid, self.ffn_out, H, self.hidden, s)
        ctx.rms_norm_rows(self.hidden, self._vec("output_norm.weight"), 1, H, cfg.eps, self.normed, s)
        out = "output.weight" if "output.weight" in self.w else "token_embd.weight"
        self._project([(out, self.normed, self.logits)], s)
        ctx.argmax(self.logits, self.key, 0, s)
        ctx.token_commit(self.key, self.prompt, n_prompt, self.pos, self.next_id, self.tokens, self.max_new, s)

    # ---------------------------------------------------------------- control
    def reset(self) -> None:
        """Empty caches and states, position 0 (HybridCache::reset)."""
        with self.torch.cuda.stream(self.stream):
            for t in (*self.keys.values(), *self.values.values(), *self.hist.values(), *self.state.values()):
                t.zero_()
            self.pos.zero_()
            self.tokens.zero_()
        self.stream.synchronize()

    def capture(self, n_prompt: int) -> None:
        """Capture the step in a CUDA graph (after one uncaptured warm-up step
        that sizes every scratch buffer; the state is reset afterwards)."""
        torch = self.torch
        s = self.stream
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
        """Replay one captured step on the decoder's stream (asynchronous)."""
        with self.torch.cuda.stream(self.stream):
            self.graph.replay()

    def start(self, prompt) -> None:
        """Reset and load a prompt; the next step ingests prompt[0]."""
        torch = self.torch
        prompt = np.ascontiguousarray(prompt, np.uint32)
        if prompt.size == 0 or prompt.size > self.cap:
            raise ValueError("prompt must hold 1 .. capacity tokens")
        if self.graph is None or self.graph_prompt != prompt.size:
            self.capture(int(prompt.size))
        self.reset()
        with torch.cuda.stream(self.stream):
            self.prompt[:prompt.size].copy_(torch.from_numpy(prompt.view(np.int32)).to(self.dev, non_blocking=False))
            self.next_id.fill_(int(prompt[0]))
        self.stream.synchronize()

    def generate(self, prompt, n_new: int) -> np.ndarray:
        """Fresh greedy generation: n_new tokens after the prompt
        (Qwen35GenerationSession::generate_fresh at temperature 0)."""
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
        """One step on `token` at the current position; returns the logits."""
        if self.graph is None:
            self.capture(1)
        with self.torch.cuda.stream(self.stream):
            self.next_id.fill_(int(token))
            self.graph.replay()
        self.stream.synchronize()
        self.ctx.device_status()
        return self.logits.cpu().numpy().copy()

    def profile_projections(self) -> tuple:
        """One uncaptured step with CUDA events around every projection call:
        (weight bytes streamed by the projections, their summed milliseconds,
        the whole step's milliseconds).  The state is reset afterwards."""
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

    def close(self) -> None:
        """Release the graph and the peer group (before the process group goes)."""
        self.graph = None
        if self.group is not None:
            self.stream.synchronize()
            self.group.close()
            self.group = None

    def launches_per_step(self) -> int:
        """Kernels one step launches (counted by the context on an uncaptured step)."""
        before = self.ctx.launch_count()
        self._enqueue_step(self.graph_prompt or 1, self.stream.cuda_stream)
        self.stream.synchronize()
        n = self.ctx.launch_count() - before
        self.reset()
        return n
