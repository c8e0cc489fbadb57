"""Qwen3 decode engine on the B200 decode-attention step.

Keeps the reference engine's surface (GodRishUniverse/kernel_optim engine/engine.py):

* ``Engine(model_path)`` (engine.py:119-161) loads the checkpoint with Transformers
  (bf16, attn_implementation="sdpa", local_files_only) and concatenates each layer's q/k/v weights
  into one QKV weight (engine.py:148).
* ``generate(input_ids, max_new_tokens)`` (engine.py:418-523) yields ``max_new_tokens`` lists of B
  token ids, greedy, never stopping at EOS.

What changes is the decode step (engine.py:313-341, 388-401): the per-layer ``qk_norm_rope`` +
``attn1`` pair becomes one ``PagedDecodeAttention`` launch over a paged KV cache, and the whole step
is captured once per shape in a CUDA graph and replayed, pipelined one step ahead of the host as in
engine.py:509-533. Around it the layer runs as engine.py:325-340 does, on the tcgen05 skinny GEMM
(``Gemv``, engine.py:259-263) against fused weights (q/k/v; gate and up): each RMSNorm a row kernel
(``add_rms_norm``), the down_proj residual add, SwiGLU and the LM head's greedy pick as epilogues,
o_proj a cuBLAS GEMM whose residual add the next norm takes, all in Transformers' cast order
(batches above 64 rows: cuBLAS GEMMs, ``add_rms_norm`` and ``silu_mul``). Prefill
(``prefill="native"``) runs the same row kernels over the whole prompt with cuBLAS GEMMs; the
prologue kernel writes the prompt's K/V into the pages and the tcgen05 prefill kernel attends from
there (sharded: torch SDPA over all heads); ``prefill="transformers"`` uses the native
Transformers forward.

Multi-GPU (``group`` = a torch.distributed process group of G ranks, one GPU each, one node): rank r
keeps kv heads [r*nkv/G, (r+1)*nkv/G) — their QKV weight rows and their pages — and runs attention
for them with the all-gather fused into the kernel (kernel_optim_b200/gather.py): every rank's rows
land in every rank's [B, nq*128] buffer over NVLink, which feeds o_proj directly; everything after
attention is replicated, so every rank emits the same tokens. Failures are handled on the host
between steps (comm.PeerWatch in ``generate``) and by the kernel's bounded flag wait.
"""

from __future__ import annotations

import os

import torch

from ._lib import KoptError, dev_error_text
from .comm import PeerFailure, PeerWatch
from .paged import PAGE, PagedDecodeAttention, PagedKVCache, qk_norm_rope_paged
from .fused import add_rms_norm, qk_norm_rope, silu_mul
from .prefill import prefill_attention
from .gather import PeerGather, slot_of
from .gemv import EPI_ARGMAX, EPI_BF16, EPI_RESID, EPI_SWIGLU, Gemv
from .shard import head_range, shard_qkv_weight
from .spec import HOST_MS, draft_len, drain_one_token, speculate


class Engine:
    def __init__(self, model_path: str, device: str = "cuda:0", group=None, overlap: bool = True,
                 gemv: bool = True, prefill: str = "native", spec: bool | None = None):
        from transformers import AutoModelForCausalLM
        model = AutoModelForCausalLM.from_pretrained(
            model_path, dtype=torch.bfloat16, attn_implementation="sdpa", local_files_only=True)
        self._init(model.eval().to(device), device, group, overlap, gemv, prefill, spec)

    @classmethod
    def from_model(cls, model, device: str = "cuda:0", group=None, overlap: bool = True,
                   gemv: bool = True, prefill: str = "native", spec: bool | None = None) -> "Engine":
        """Wrap an already loaded Qwen3ForCausalLM (bf16, sdpa) instead of reading a checkpoint."""
        self = cls.__new__(cls)
        self._init(model.eval().to(device), device, group, overlap, gemv, prefill, spec)
        return self

    # ------------------------------------------------------------------ construction
    def _init(self, model, device, group, overlap=True, gemv=True, prefill="native", spec=None):
        """spec: speculative decoding with n-gram drafts and the T > 1 verify step (spec.py); by
        default ENGINE_SPEC=1 turns it on and ENGINE_MIN_ADVANCE overrides the measured
        break-even, as in the reference (engine.py:38-45). One GPU only (the fused gather is
        T = 1)."""
        if prefill not in ("native", "transformers"):
            raise KoptError("prefill must be 'native' or 'transformers'")
        self.prefill = prefill
        torch.backends.cuda.matmul.allow_tf32 = False
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise KoptError("Engine needs a CUDA device (the decode step has no CPU path)")
        cfg = model.config
        self.nq, self.nkv = cfg.num_attention_heads, cfg.num_key_value_heads
        self.d = getattr(cfg, "head_dim", None) or cfg.hidden_size // self.nq
        if self.d != 128 or self.nq != 4 * self.nkv:
            raise KoptError("the decode-attention kernel needs head_dim 128 and 4 query heads per kv head")
        self.eps = cfg.rms_norm_eps
        self.n_layers = cfg.num_hidden_layers
        self.model = model
        self.group = group
        self.overlap = overlap
        self.use_gemv = gemv
        self.world = 1 if group is None else torch.distributed.get_world_size(group)
        self.rank = 0 if group is None else torch.distributed.get_rank(group)
        # failure records only: between generate calls a live rank may sit idle for any time, so
        # a peer that is gone shows instead as the fused gather's timeout in the error word
        self.watch = PeerWatch(group, stale_s=None) if self.world > 1 else None
        self.spec = (os.environ.get("ENGINE_SPEC", "0") == "1") if spec is None else bool(spec)
        self.spec = self.spec and self.world == 1
        ma = os.environ.get("ENGINE_MIN_ADVANCE")
        self.min_advance = float(ma) if ma is not None else None
        h0, _ = head_range(self.nkv, self.rank, self.world)
        self.nkv_l = self.nkv // self.world
        self.nq_l = 4 * self.nkv_l
        self.h0 = h0
        base = model.model
        self.embed = base.embed_tokens.weight
        self.layers = []
        with torch.no_grad():
            for layer in base.layers:
                a = layer.self_attn
                mlp = layer.mlp
                self.layers.append(dict(
                    mod=layer,
                    # this rank's q/k/v rows in one weight, as engine.py:148 fuses them
                    qkv=shard_qkv_weight(a.q_proj.weight, a.k_proj.weight, a.v_proj.weight,
                                         self.nkv, self.rank, self.world, self.d),
                    q_norm=a.q_norm.weight.contiguous(),
                    k_norm=a.k_norm.weight.contiguous(),
                    o=a.o_proj.weight,
                    # gate rows then up rows, the layout silu_mul reads (engine.py:150)
                    gu=torch.cat([mlp.gate_proj.weight, mlp.up_proj.weight], 0).contiguous(),
                    down=mlp.down_proj.weight,
                    w_in=layer.input_layernorm.weight.contiguous(),
                    w_post=layer.post_attention_layernorm.weight.contiguous(),
                ))
            self.final_norm = base.norm.weight.contiguous()
            self.inter = base.layers[0].mlp.gate_proj.weight.shape[0]
        self._shape = None
        self.graph = None
        self.pg = None

    def _rope(self, n):
        pos = torch.arange(n, device=self.device).unsqueeze(0)
        dummy = torch.empty(1, dtype=torch.bfloat16, device=self.device)
        cos, sin = self.model.model.rotary_emb(dummy, pos)   # exactly the native tables
        return cos[0].contiguous(), sin[0].contiguous()

    def _setup(self, B, S, N):
        if self._shape == (B, S, N):
            return
        self.graph = None
        self.gk = None
        self._shape = None
        self.K = draft_len(B) if self.spec and N > 2 else 0
        # speculating, a sequence can run ahead of the slowest one by up to N + K tokens
        cap = S + 2 * N + 2 * self.K + 2 if self.K else S + N + 1
        self.cos, self.sin = self._rope(cap)
        pages = B * ((cap + PAGE - 1) // PAGE)
        self.cache = PagedKVCache(self.n_layers, pages, self.nkv_l, self.d, B, cap, self.device)
        self.cache.assign_sequential([cap] * B)
        # the kernel before each attention call is the QKV projection GEMM, which writes neither
        # positions, block table nor cache: the call may start while it finishes
        self.attn = PagedDecodeAttention(B, self.nq_l, self.nkv_l, self.d, self.device,
                                         self.cache.capacity, eps=self.eps,
                                         overlap_prev=self.overlap)
        self.B, self.S, self.cap = B, S, cap
        dev, bf = self.device, torch.bfloat16
        self.ids = torch.zeros(B, dtype=torch.int64, device=dev)
        self.pos = torch.zeros(B, dtype=torch.int32, device=dev)
        self.attn_out = torch.zeros(B, self.nq_l * self.d, dtype=bf, device=dev)
        H = self.embed.shape[1]
        self.hid = torch.zeros(B, H, dtype=bf, device=dev)       # residual stream
        self.normed = torch.zeros(B, H, dtype=bf, device=dev)
        self.act = torch.zeros(B, self.inter, dtype=bf, device=dev)
        self.gemv = None
        if self.use_gemv and B <= 64:   # the skinny-GEMM kernel serves up to 64 rows
            nqkv = self.layers[0]["qkv"].shape[0]
            ov = self.overlap
            self.qkv = torch.zeros(B, nqkv, dtype=bf, device=dev)
            # each RMSNorm is a row kernel writing the normalised rows once; the projections read
            # them (normalising inside the projection, kopt_gemv_fused, measured slower here)
            # o_proj (K = 4096 against N = 2560: a 20-tile weight split seven ways along K) stays
            # on cuBLAS, its residual add folded into the post-attention norm: with the skinny-GEMM
            # kernel there, with or without the overlap of the attention, a Qwen3-4B decode step at
            # B = 32 took 4.02-4.07 ms against 3.83 ms
            self.gemv = dict(
                qkv=Gemv(B, nqkv, H, EPI_BF16, device=dev, overlap_prev=ov),
                gu=Gemv(B, self.inter, H, EPI_SWIGLU, device=dev, overlap_prev=ov),
                down=Gemv(B, H, self.inter, EPI_RESID, device=dev, overlap_prev=ov),
            )
            lm_w = self.model.lm_head.weight
            if lm_w.shape[0] % 64 == 0 and lm_w.is_contiguous():
                # LM head + greedy pick in one kernel: token ids, no logits in HBM
                self.gemv["lm"] = Gemv(B, lm_w.shape[0], H, EPI_ARGMAX, device=dev, overlap_prev=ov)
        if self.pg is not None:
            self.pg.close()
            self.pg = None
        if self.world > 1:
            self.pg = PeerGather(B, self.nq * self.d, dev, self.group)
        self.pin_ids = torch.empty(N + 1, B, dtype=torch.int64, pin_memory=True)
        # sharded: the attention's error word after each step, read back beside the token ids
        self.pin_err = (torch.zeros(N + 1, dtype=torch.int32, pin_memory=True)
                        if self.watch is not None else None)
        self.events = [torch.cuda.Event() for _ in range(N + 1)]
        self.pin_pos = torch.empty(B, dtype=torch.int32, pin_memory=True)
        self.graph = self._capture(self._step)
        if self.K:
            self._setup_verify(B, S)
        self._shape = (B, S, N)

    def _setup_verify(self, B, S):
        """The verify step's buffers, plan and graph, and the break-even advance per verify step
        (engine.py:209-223): measured from the two graphs unless ENGINE_MIN_ADVANCE is set."""
        T, dev, bf = self.K + 1, self.device, torch.bfloat16
        M, H = B * T, self.embed.shape[1]
        self.attnk = PagedDecodeAttention(B, self.nq_l, self.nkv_l, self.d, dev, self.cache.capacity,
                                          eps=self.eps, T=T)
        self.vin = torch.zeros(B, T, dtype=torch.int64, device=dev)
        self.vout = torch.zeros(B, T, dtype=torch.int64, device=dev)
        self.pin_vin = torch.empty(B, T, dtype=torch.int64, pin_memory=True)
        self.pin_vout = torch.empty(B, T, dtype=torch.int64, pin_memory=True)
        self.hid_k = torch.zeros(M, H, dtype=bf, device=dev)
        self.normed_k = torch.zeros(M, H, dtype=bf, device=dev)
        self.q_k = torch.zeros(M, self.nq_l * self.d, dtype=bf, device=dev)
        self.out_k = torch.zeros(M, self.nq_l * self.d, dtype=bf, device=dev)
        self.act_k = torch.zeros(M, self.inter, dtype=bf, device=dev)
        self.ev_k = torch.cuda.Event()
        self.gk = self._capture(self._stepk)
        t1, tk = self._time_graph(self.graph, S), self._time_graph(self.gk, S)
        self.breakeven = (tk + HOST_MS) / t1 if self.min_advance is None else self.min_advance
        self.step_ms, self.verify_ms = t1, tk

    def _time_graph(self, g, S, reps=10):
        """ms per replay, from a position where every write stays inside the cache."""
        start = max(0, min(S, self.cap - (reps + 2) - (self.K + 1)))
        torch.cuda.synchronize(self.device)
        self.pos.fill_(start)
        g.replay()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            g.replay()
        b.record()
        torch.cuda.synchronize(self.device)
        return a.elapsed_time(b) / reps

    def _capture(self, fn):
        # warm up on a side stream (cuBLAS handles, kernel attributes), then capture once
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            for _ in range(2):
                self.pos.fill_(1)
                fn()
        torch.cuda.current_stream(self.device).wait_stream(s)
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        self.pos.fill_(1)
        with torch.cuda.graph(g):
            fn()
        torch.cuda.synchronize(self.device)
        return g

    # ----------------------------------------------------------------------- forward
    def _attention(self, i, lw, qkv):
        """Attention of layer i; returns [B, nq*128] (all heads, gathered when sharded)."""
        if self.pg is None:
            self.attn(qkv, lw["q_norm"], lw["k_norm"], self.cos, self.sin, self.cache, i, self.pos,
                      self.attn_out)
            return self.attn_out
        return self.pg.attend(self.attn, qkv, lw["q_norm"], lw["k_norm"], self.cos, self.sin,
                              self.cache, i, self.pos, slot_of(i, self.n_layers))

    def _step(self):
        """One decode step at positions pos[b]; argmax feeds ids, positions advance. The layer
        loop of engine.py:325-340. With the skinny-GEMM kernels (B <= 64) the down_proj residual
        add, SwiGLU and the greedy pick are the projections' epilogues (gemv.py:86-105), o_proj a
        cuBLAS GEMM whose residual add the post-attention norm takes, and each RMSNorm a row
        kernel; otherwise cuBLAS GEMMs with the residual add fused into the next RMSNorm."""
        h, n = self.hid, self.normed
        torch.index_select(self.embed, 0, self.ids, out=h)
        gv = self.gemv
        if gv is not None:
            for i, lw in enumerate(self.layers):
                add_rms_norm(h, None, lw["w_in"], n, self.eps)
                gv["qkv"](n, lw["qkv"], self.qkv)
                o = torch.mm(self._attention(i, lw, self.qkv), lw["o"].t())
                add_rms_norm(h, o, lw["w_post"], n, self.eps)
                gv["gu"](n, lw["gu"], self.act)
                gv["down"](self.act, lw["down"], h=h)
            add_rms_norm(h, None, self.final_norm, n, self.eps)
            if "lm" in gv:
                gv["lm"](n, self.model.lm_head.weight, self.ids)
                self.pos.add_(1)
                return
        else:
            delta = None
            for i, lw in enumerate(self.layers):
                add_rms_norm(h, delta, lw["w_in"], n, self.eps)
                qkv = torch.mm(n, lw["qkv"].t())
                o = torch.mm(self._attention(i, lw, qkv), lw["o"].t())
                add_rms_norm(h, o, lw["w_post"], n, self.eps)
                silu_mul(torch.mm(n, lw["gu"].t()), self.act)
                delta = torch.mm(self.act, lw["down"].t())
            add_rms_norm(h, delta, self.final_norm, n, self.eps)
        logits = self.model.lm_head(n)
        torch.argmax(logits, dim=-1, out=self.ids)
        self.pos.add_(1)

    def _stepk(self):
        """Verify step (engine.py:403-415): rows vin[b] = the last accepted token and K drafts at
        positions pos[b] .. pos[b] + K; vout[b] = the greedy pick after each. The layer loop of the
        cuBLAS decode step over B (K + 1) rows, with the prologue appending the K + 1 tokens' K/V
        to the pages (kopt_qk_norm_rope, T = K + 1) and the T > 1 verify attention
        (kopt_decode_attn), each query row seeing the keys up to its own position."""
        T = self.K + 1
        h, n = self.hid_k, self.normed_k
        torch.index_select(self.embed, 0, self.vin.view(-1), out=h)
        delta = None
        for i, lw in enumerate(self.layers):
            add_rms_norm(h, delta, lw["w_in"], n, self.eps)
            qkv = torch.mm(n, lw["qkv"].t())
            qk_norm_rope_paged(qkv, lw["q_norm"], lw["k_norm"], self.cos, self.sin, self.pos, self.q_k,
                               self.cache, i, T, self.eps, self.nq_l, self.nkv_l, self.d)
            self.attnk.attend(self.q_k, self.cache, i, self.pos, self.out_k)
            add_rms_norm(h, torch.mm(self.out_k, lw["o"].t()), lw["w_post"], n, self.eps)
            silu_mul(torch.mm(n, lw["gu"].t()), self.act_k)
            delta = torch.mm(self.act_k, lw["down"].t())
        add_rms_norm(h, delta, self.final_norm, n, self.eps)
        torch.argmax(self.model.lm_head(n), dim=-1, out=self.vout.view(-1))

    def _verify(self, rows, positions):
        """One verify forward from the host: rows [B][K + 1] at positions [B]; the picks back."""
        stream = torch.cuda.current_stream(self.device)
        self.pin_vin.copy_(torch.tensor(rows, dtype=torch.int64))
        self.pin_pos.copy_(torch.tensor(positions, dtype=torch.int32))
        self.vin.copy_(self.pin_vin, non_blocking=True)
        self.pos.copy_(self.pin_pos, non_blocking=True)
        self.gk.replay()
        self.pin_vout.copy_(self.vout, non_blocking=True)
        self.ev_k.record(stream)
        self.ev_k.synchronize()
        self.spec_steps += 1
        return self.pin_vout.tolist()

    def _qkv_full(self, i):
        """Layer i's QKV weight for all heads (prefill attends with every head on every rank)."""
        lw = self.layers[i]
        if self.world == 1:
            return lw["qkv"]
        if "qkv_full" not in lw:
            a = lw["mod"].self_attn
            lw["qkv_full"] = torch.cat([a.q_proj.weight, a.k_proj.weight, a.v_proj.weight], 0).contiguous()
        return lw["qkv_full"]

    def _prefill(self, prompt):
        if self.prefill == "native":
            self._prefill_native(prompt)
        else:
            self._prefill_transformers(prompt)

    def _prefill_native(self, prompt):
        """Prefill on the row kernels of the decode step, Qwen3DecoderLayer's cast order: per layer
        the residual add + input RMSNorm (add_rms_norm), one QKV GEMM, the q/k RMSNorm + RoPE
        prologue (kopt_qk_norm_rope), causal GQA attention, o_proj, residual add +
        post-attention RMSNorm, gate|up GEMM, SwiGLU (silu_mul), down_proj. On one GPU the prologue
        writes the prompt's K/V straight into the pages and the attention is the tcgen05 prefill
        kernel reading them there (kopt_prefill_attn); sharded, every rank attends with all heads
        (torch SDPA on the prologue's K/V) and keeps its own kv heads' K/V in its pages. Only the
        last position goes through the final norm and the LM head (the reference's prefill keeps
        only its logits too)."""
        B, S = prompt.shape
        H, nq, nkv, d = self.embed.shape[1], self.nq, self.nkv, self.d
        dev, bf, M = self.device, torch.bfloat16, B * S
        h = torch.index_select(self.embed, 0, prompt.reshape(-1))
        n = torch.empty_like(h)
        q = torch.empty(M, nq * d, dtype=bf, device=dev)
        if self.world > 1:   # sharded: every head's K/V, for the all-head attention
            k = torch.empty(B, nkv, S, d, dtype=bf, device=dev)
            v = torch.empty_like(k)
        act = torch.empty(M, self.inter, dtype=bf, device=dev)
        pos0 = torch.zeros(B, dtype=torch.int32, device=dev)
        h0 = self.h0
        delta = None
        attn = torch.empty(M, nq * d, dtype=bf, device=dev) if self.world == 1 else None
        for i, lw in enumerate(self.layers):
            add_rms_norm(h, delta, lw["w_in"], n, self.eps)
            qkv = torch.mm(n, self._qkv_full(i).t())
            if self.world == 1:
                qk_norm_rope_paged(qkv, lw["q_norm"], lw["k_norm"], self.cos, self.sin, pos0, q,
                                   self.cache, i, S, self.eps, nq, nkv, d)
                prefill_attention(q, self.cache, i, attn, B, S, nq, nkv, d)
                o = torch.mm(attn, lw["o"].t())
            else:
                qk_norm_rope(qkv, lw["q_norm"], lw["k_norm"], self.cos, self.sin, pos0, q, k, v, S,
                             self.eps, nq, nkv, d)
                a = torch.nn.functional.scaled_dot_product_attention(
                    q.view(B, S, nq, d).transpose(1, 2), k, v, is_causal=True, enable_gqa=True)
                o = torch.mm(a.transpose(1, 2).reshape(M, nq * d), lw["o"].t())
                self.cache.write_prefix(i, k[:, h0:h0 + self.nkv_l], v[:, h0:h0 + self.nkv_l])
            add_rms_norm(h, o, lw["w_post"], n, self.eps)
            silu_mul(torch.mm(n, lw["gu"].t()), act)
            delta = torch.mm(act, lw["down"].t())
        last = h.view(B, S, H)[:, -1].contiguous()
        nl = torch.empty_like(last)
        add_rms_norm(last, delta.view(B, S, H)[:, -1].contiguous(), self.final_norm, nl, self.eps)
        self.ids.copy_(self.model.lm_head(nl).argmax(dim=-1))
        self.pos.fill_(S)

    def _prefill_transformers(self, prompt):
        """The native forward over the prompt; its K/V (this rank's heads) go into the pages."""
        out = self.model(input_ids=prompt, use_cache=True)
        self.ids.copy_(out.logits[:, -1, :].argmax(dim=-1))
        h0 = self.h0
        for i, layer in enumerate(out.past_key_values.layers):
            self.cache.write_prefix(i, layer.keys[:, h0:h0 + self.nkv_l],
                                    layer.values[:, h0:h0 + self.nkv_l])
        self.pos.fill_(prompt.shape[1])

    # ---------------------------------------------------------------------- generate
    @torch.inference_mode()
    def generate(self, input_ids: list[list[int]], max_new_tokens: int):
        """Greedy tokens, one list of B ids per step. Sharded, every rank checks the group's
        failure record (comm.PeerWatch) before each decode step, records its own failure there
        when it raises, and reads the attention's device error word after every step and at the
        end (a peer that stopped shows as KOPT_DEV_ERR_TIMEOUT of the fused gather)."""
        if self.watch is None:
            yield from self._generate(input_ids, max_new_tokens)
            return
        try:
            self.watch.check()
            yield from self._generate(input_ids, max_new_tokens)
            bits = self.attn.read_error()
            if bits:
                raise KoptError(f"rank {self.rank}: device error bits {bits} ({dev_error_text(bits)})")
        except (Exception, KeyboardInterrupt) as e:
            if not isinstance(e, PeerFailure):
                self.watch.fail(f"{type(e).__name__}: {e}")
            raise

    def _generate(self, input_ids: list[list[int]], max_new_tokens: int):
        N = max_new_tokens
        if N <= 0:
            return
        B, S = len(input_ids), len(input_ids[0])
        if any(len(r) != S for r in input_ids):
            raise KoptError("prompts must have equal length")
        self._setup(B, S, N)
        stream = torch.cuda.current_stream(self.device)
        prompt = torch.tensor(input_ids, dtype=torch.int64).pin_memory().to(self.device, non_blocking=True)
        self._prefill(prompt)
        ids_h, ev = self.pin_ids, self.events
        ids_h[0].copy_(self.ids, non_blocking=True)
        ev[0].record(stream)
        self.spec_steps = 0
        if self.K:
            yield from self._generate_spec(input_ids, N, S)
            return
        # queue the next step before waiting on the current one (engine.py:509-533)
        err_h = self.pin_err
        for j in range(1, N):
            if self.watch is not None:
                self.watch.check()
            self.graph.replay()
            ids_h[j].copy_(self.ids, non_blocking=True)
            if err_h is not None:
                err_h[j:j + 1].copy_(self.attn.ws[:4].view(torch.int32), non_blocking=True)
            ev[j].record(stream)
            ev[j - 1].synchronize()
            if err_h is not None and int(err_h[j - 1]):
                bits = int(err_h[j - 1])
                raise KoptError(f"rank {self.rank}: device error bits {bits} ({dev_error_text(bits)}) "
                                f"by decode step {j - 1}")
            yield ids_h[j - 1].tolist()
        ev[N - 1].synchronize()
        yield ids_h[N - 1].tolist()

    def _generate_spec(self, input_ids, N, S):
        """Speculative generate (engine.py:451-508): verify steps while they pay for themselves,
        then the one-token graph from each sequence's own position."""
        self.events[0].synchronize()
        first = self.pin_ids[0].tolist()
        yield first
        if N == 1:
            return
        outs = yield from speculate(input_ids, first, N, self.K, self._verify, self.breakeven)
        ready = min(len(o) for o in outs)
        if ready >= N:
            return
        # hand each sequence's last token and position to the one-token graph
        self.pin_ids[0].copy_(torch.tensor([o[-1] for o in outs], dtype=torch.int64))
        self.pin_pos.copy_(torch.tensor([S + len(o) - 1 for o in outs], dtype=torch.int32))
        self.ids.copy_(self.pin_ids[0], non_blocking=True)
        self.pos.copy_(self.pin_pos, non_blocking=True)
        yield from drain_one_token(outs, N, self._one_token_steps(N - ready))

    def _one_token_steps(self, n):
        """n replays of the one-token graph, each queued before the host waits on the one before;
        yields each step's token ids."""
        stream = torch.cuda.current_stream(self.device)
        ids_h, ev = self.pin_ids, self.events
        for j in range(1, n + 1):
            self.graph.replay()
            ids_h[j].copy_(self.ids, non_blocking=True)
            ev[j].record(stream)
            if j > 1:
                ev[j - 1].synchronize()
                yield ids_h[j - 1].tolist()
        if n:
            ev[n].synchronize()
            yield ids_h[n].tolist()

    def read_error(self) -> int:
        """Device error bits of the attention kernel since the last read (synchronises)."""
        return self.attn.read_error()

    def close(self) -> None:
        """Release the cross-rank gather buffers (collective when sharded)."""
        self.graph = None
        self._shape = None
        if self.pg is not None:
            self.pg.close()
            self.pg = None
