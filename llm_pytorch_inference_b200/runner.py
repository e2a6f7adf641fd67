"""Decode-step runner: one batched decode forward + sampling on the sm_100a kernels.

Replaces the per-step body of ``LLMEngine._run_decode`` (``mini_vllm/engine/engine.py:297-360``):
the model forward of ``ForCausalLM`` (``models/model.py:412-424``) for one new token
per sequence over the paged KV pool, then ``Sampler.sample`` for every row.

Everything the step touches is resident on the device and laid out once:

* weights in bf16, the q/k/v projections concatenated into one ``[(Hq+2Hkv)*D, H]``
  matrix per layer and gate/up into the reference's fused ``cat([gate, up])``
  (``ops/mlp.py:87-121``);
* the model's bf16 cos/sin tables, built once exactly as ``RotaryEmbedding`` builds
  them after ``model.to(bf16)`` (``models/model.py:28-81``);
* activations, logits and sampled tokens in fixed buffers;
* per-step metadata (token ids, positions, context lengths, block tables, sampling
  offset) in one int32 device buffer filled by one host->device copy per step;
* stream-K / split-KV workspaces (zero-initialised once; the kernels leave them zero).

A step is 8 kernels per layer.  ``capture()`` records the whole step in one CUDA
graph; ``replay()`` re-runs it (the host only refreshes the metadata buffer).

With tensor parallelism (``tp.tp_size > 1``, one runner per GPU) the weights are the rank's
shard (``tensor_parallel.shard_state_dict``), the KV pool holds the rank's KV heads, and the
normalised activations and the logits live in the symmetric heap that the TP kernels write
across GPUs (``tensor_parallel``).
"""
from __future__ import annotations

import math

import torch

from . import _native as N
from .configs import embed_scale, head_dim, is_gemma, layer_rope_theta, layer_window, num_kv_heads
from .kv_cache import KVCacheManager
from . import tensor_parallel as tpm
from .tensor_parallel import TensorParallelConfig


def resolve_device(device) -> torch.device:
    """``cuda`` -> ``cuda:<current>`` so device comparisons are exact."""
    dev = torch.device(device)
    if dev.type == "cuda" and dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    return dev


def rope_tables(head_dim_: int, theta: float, length: int, dtype: torch.dtype, device) -> tuple[torch.Tensor, torch.Tensor]:
    """cos/sin ``[length, D]`` as the reference's ``RotaryEmbedding`` holds them after
    ``model.to(dtype)``: fp32 ``inv_freq`` rounded to ``dtype``, position ramp in ``dtype``
    (``models/model.py:31``, ``:75-80``).  Built on ``device``, as the reference builds them on the
    device of the positions: a bf16 ramp rounds differently on the CPU and on the GPU past
    position 4112, and a bf16 model decodes on the GPU."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim_, 2).float() / head_dim_))
    inv = inv.to(dtype).to(device)
    t = torch.arange(length, dtype=inv.dtype, device=device)
    freqs = torch.outer(t, inv)
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos().contiguous(), emb.sin().contiguous()


def meta_layout(batch: int, max_blocks: int) -> dict[str, int]:
    """Offsets (in int32 words) of the per-step metadata buffer, one upload per step:
    token ids | positions | context lengths | sampling offset (int64, 8-byte aligned) |
    temperature (fp32) | top-k (int32) | top-p (fp32) | feed (int32: nonzero = take the ids from
    the previous step's sampled tokens on the device) | block tables ``[batch, max_blocks]``."""
    B = batch
    o_off = (3 * B + 1) // 2 * 2
    o_temp = o_off + 2
    o_topk = o_temp + B
    o_topp = o_topk + B
    o_feed = o_topp + B
    o_bt = o_feed + 1
    return {"ids": 0, "pos": B, "ctx": 2 * B, "off": o_off, "temp": o_temp, "topk": o_topk, "topp": o_topp,
            "feed": o_feed, "bt": o_bt, "total": o_bt + B * max_blocks}


class DecodeWeights:
    """Per-layer device weights in the layout the decode kernels read."""

    def __init__(self, cfg: dict, sd: dict[str, torch.Tensor], device, dtype=torch.bfloat16):
        L = cfg["num_hidden_layers"]
        dev = resolve_device(device)

        def get(k):
            return sd[k].to(device=dev, dtype=dtype).contiguous()

        self.embed = get("model.embed_tokens.weight")
        self.lm_head = get("lm_head.weight") if "lm_head.weight" in sd else self.embed
        self.final_norm = get("model.norm.weight")
        self.qk_norm = cfg.get("_qk_norm", False)
        self.wqkv, self.wo, self.wgu, self.wdown, self.ln1, self.ln2, self.qn, self.kn = ([] for _ in range(8))
        self.pre_ff, self.post_ff = [], []   # Gemma: pre/post feed-forward norms (gemma3_model.py:265-268)
        self.moe = bool(cfg.get("num_experts"))
        self.router, self.egu, self.edown = [], [], []    # MoE: [E, H], [E, 2I, H], [E, H, I]
        for i in range(L):
            p = f"model.layers.{i}."
            a = p + "self_attn."
            self.wqkv.append(torch.cat([get(a + "q_proj.weight"), get(a + "k_proj.weight"),
                                        get(a + "v_proj.weight")], 0).contiguous())
            self.wo.append(get(a + "o_proj.weight"))
            if self.moe:
                self.router.append(get(p + "mlp.gate.weight"))
                e = p + "mlp.experts."
                if e + "gate_up_proj.weight" in sd:
                    self.egu.append(get(e + "gate_up_proj.weight"))
                    self.edown.append(get(e + "down_proj.weight"))
                else:
                    E = 0   # the experts this GPU holds (all, or a tensor-parallel rank's share)
                    while f"{e}{E}.gate_proj.weight" in sd:
                        E += 1
                    self.egu.append(torch.stack([torch.cat([get(f"{e}{j}.gate_proj.weight"), get(f"{e}{j}.up_proj.weight")],
                                                           0) for j in range(E)]).contiguous())
                    self.edown.append(torch.stack([get(f"{e}{j}.down_proj.weight") for j in range(E)]).contiguous())
            elif p + "mlp.gate_up_proj.weight" in sd:   # already fused (ops/mlp.py:87-121)
                self.wgu.append(get(p + "mlp.gate_up_proj.weight"))
                self.wdown.append(get(p + "mlp.down_proj.weight"))
            else:
                self.wgu.append(torch.cat([get(p + "mlp.gate_proj.weight"), get(p + "mlp.up_proj.weight")],
                                          0).contiguous())
                self.wdown.append(get(p + "mlp.down_proj.weight"))
            self.ln1.append(get(p + "input_layernorm.weight"))
            self.ln2.append(get(p + "post_attention_layernorm.weight"))
            if cfg.get("_has_feedforward_layernorms"):
                self.pre_ff.append(get(p + "pre_feedforward_layernorm.weight"))
                self.post_ff.append(get(p + "post_feedforward_layernorm.weight"))
            if self.qk_norm:
                self.qn.append(get(a + "q_norm.weight"))
                self.kn.append(get(a + "k_norm.weight"))

    def nbytes(self) -> int:
        ts = [self.embed, self.final_norm, *self.wqkv, *self.wo, *self.wgu, *self.wdown, *self.ln1, *self.ln2,
              *self.qn, *self.kn, *self.router, *self.egu, *self.edown, *self.pre_ff, *self.post_ff]
        if self.lm_head is not self.embed:
            ts.append(self.lm_head)
        return sum(t.numel() * t.element_size() for t in ts)

    def streamed_bytes(self) -> int:
        """Weight bytes one decode step must read: every layer's matrices and norms, the final norm
        and lm_head (the embedding table is only gathered, one row per sequence)."""
        ts = [self.final_norm, self.lm_head, *self.wqkv, *self.wo, *self.wgu, *self.wdown, *self.ln1, *self.ln2,
              *self.qn, *self.kn, *self.router, *self.egu, *self.edown, *self.pre_ff, *self.post_ff]
        return sum(t.numel() * t.element_size() for t in ts)


class DecodeRunner:
    def __init__(self, cfg: dict, weights: DecodeWeights, kv: KVCacheManager, max_batch: int, max_model_len: int,
                 device="cuda", rope_len: int | None = None, tp: TensorParallelConfig | None = None,
                 fused_layers: bool = False):
        """``fused_layers``: run each layer after its attention as one persistent launch
        (``mvb_decoder_layer_tail``; dense, one GPU, batch <= 64, head dim 128, hidden <= 4096)
        instead of the per-kernel step.  Off by default: on B200 the per-kernel step with
        programmatic dependent launch is the faster of the two at Qwen3-8B dims."""
        self.cfg = cfg
        self.w = weights
        self.kv = kv
        self.dev = resolve_device(device)
        self.tp = tp or TensorParallelConfig()
        T = self.tp.tp_size
        tpm.check_divisible(cfg, T)
        if max_batch % T:
            raise ValueError(f"max_batch {max_batch} must be a multiple of tp_size {T}")
        self.B = max_batch
        self.L = cfg["num_hidden_layers"]
        self.H = cfg["hidden_size"]
        self.Hq = cfg["num_attention_heads"] // T       # this rank's heads / features
        self.Hkv = tpm.local_kv_heads(cfg, T)   # one replicated head when there are fewer than ranks
        self.D = head_dim(cfg)
        self.I = cfg["intermediate_size"] // T
        self.V = cfg["vocab_size"]                       # full vocabulary (logits are all-gathered)
        self.Vl = self.V // T
        self.eps = float(cfg.get("rms_norm_eps", 1e-6))
        self.scale = 1.0 / math.sqrt(cfg.get("query_pre_attn_scalar") or self.D)
        if kv.kv_cache is None or kv.kv_cache.device != self.dev or kv.kv_cache.dtype != torch.bfloat16:
            raise RuntimeError("DecodeRunner needs a bf16 KV pool on the runner's device")
        if kv.block_size != 16 or kv.head_dim != self.D or kv.num_heads != self.Hkv or kv.num_layers != self.L:
            raise RuntimeError("KV pool geometry does not match the model")
        self.max_blocks = (max_model_len + kv.block_size - 1) // kv.block_size
        self.P = kv.kv_cache.shape[2]  # includes the scratch block
        rope_len = rope_len or max(max_model_len, 256)
        # Gemma: sandwich (1 + w) norms, GeGLU, scaled embedding, per-layer RoPE theta and window,
        # soft-capped attention / final logits (0 = off).
        self.gemma = is_gemma(cfg)
        self.plus_one = 1 if (self.gemma or cfg.get("_rms_norm_plus_one")) else 0
        self.act = N.ACT_GELU_TANH if cfg.get("hidden_act") in ("gelu_new", "gelu_pytorch_tanh") else N.ACT_SILU
        self.embed_scale = embed_scale(cfg)
        self.softcap = float(cfg.get("attn_logit_softcapping") or 0.0)
        self.final_softcap = float(cfg.get("final_logit_softcapping") or 0.0)
        self.windows = [layer_window(cfg, i) for i in range(self.L)]
        self.tables = {}
        for i in range(self.L):
            th = layer_rope_theta(cfg, i)
            if th not in self.tables:
                self.tables[th] = rope_tables(self.D, th, rope_len, torch.bfloat16, self.dev)
        self.layer_tables = [self.tables[layer_rope_theta(cfg, i)] for i in range(self.L)]
        self.cos, self.sin = self.layer_tables[0]

        B, H, dev, bf = self.B, self.H, self.dev, torch.bfloat16
        qkv_n = (self.Hq + 2 * self.Hkv) * self.D
        didx = dev.index if dev.index is not None else torch.cuda.current_device()
        self.heap = None
        self.residual = torch.zeros(B, H, dtype=bf, device=dev)
        if self.tp.enabled:
            lib = N.lib()
            recv_o = lib.mvb_tp_recv_bytes(B, H, self.Hq * self.D, T, didx)
            # down_proj partials; a sparse MoE block pushes one combined partial per rank (one k-block plan)
            recv_d = lib.mvb_tp_recv_bytes(B, H, 64 if cfg.get("num_experts") else self.I, T, didx)
            self.layout = tpm.plan_heap(lib.mvb_tp_signal_bytes(), B, H, self.V, recv_o, recv_d)
            self.heap = tpm.SymmetricHeap(self.layout.total, self.tp.rank, T)
            self.xn = self.heap.tensor(self.layout.xn, (B, H), bf, dev)
            self.logits = self.heap.tensor(self.layout.logits, (B, self.V), bf, dev)
        else:
            self.xn = torch.zeros(B, H, dtype=bf, device=dev)
            self.logits = torch.zeros(B, self.V, dtype=bf, device=dev)
        self.q = torch.zeros(B, self.Hq, self.D, dtype=bf, device=dev)
        self.attn = torch.zeros(B, self.Hq * self.D, dtype=bf, device=dev)
        self.h = torch.zeros(B, self.I, dtype=bf, device=dev)
        self.moe = bool(cfg.get("num_experts"))
        if self.moe:
            self.E, self.K = cfg["num_experts"], cfg["num_experts_per_tok"]
            # expert parallel under tensor parallelism: this rank's experts (all of them on one GPU)
            self.e_first, self.e_local = (tpm.expert_range(cfg, T, self.tp.rank) if self.tp.enabled else (0, self.E))
            self.Im = cfg["moe_intermediate_size"]
            self.norm_topk = 1 if cfg.get("norm_topk_prob", True) else 0
            i32 = torch.int32
            self.router_logits = torch.zeros(B, self.E, dtype=bf, device=dev)
            self.topk_ids = torch.zeros(B, self.K, dtype=i32, device=dev)
            self.topk_w = torch.zeros(B, self.K, dtype=torch.float32, device=dev)
            self.pair_row = torch.zeros(B, self.K, dtype=i32, device=dev)
            self.row_token = torch.zeros(B * self.K, dtype=i32, device=dev)
            self.expert_off = torch.zeros(self.E + 1, dtype=i32, device=dev)
            self.active = torch.zeros(self.E + 1, dtype=i32, device=dev)
            self.x_sorted = torch.zeros(B * self.K, H, dtype=bf, device=dev)
            self.h_sorted = torch.zeros(B * self.K, self.Im, dtype=bf, device=dev)
            self.y_sorted = torch.zeros(B * self.K, H, dtype=bf, device=dev)
            self.mlp_out = torch.zeros(B, H, dtype=bf, device=dev)
        self.tokens = torch.zeros(B, dtype=torch.int64, device=dev)
        self.seed = 0
        self.probs = None   # [B, V] fp32 filtered / tempered probabilities, when requested (set_probs_out)

        # metadata: ids | pos | ctx | offset(int64) | temperature | top-k | top-p | block tables
        lay = meta_layout(B, self.max_blocks)
        self.meta_offsets = lay
        self._o_pos, self._o_ctx, self._o_off, self._o_bt = lay["pos"], lay["ctx"], lay["off"], lay["bt"]
        self.meta = torch.zeros(lay["total"], dtype=torch.int32, device=dev)
        self.meta_host = torch.zeros(lay["total"], dtype=torch.int32, pin_memory=True)
        self.ids = self.meta[0:B]
        self.pos = self.meta[self._o_pos:self._o_pos + B]
        self.ctx = self.meta[self._o_ctx:self._o_ctx + B]
        self.offset = self.meta[self._o_off:self._o_off + 2].view(torch.int64)
        # per-row sampling parameters travel with the step's metadata (greedy by default)
        self.temperature = self.meta[lay["temp"]:lay["temp"] + B].view(torch.float32)
        self.top_k = self.meta[lay["topk"]:lay["topk"] + B]
        self.top_p = self.meta[lay["topp"]:lay["topp"] + B].view(torch.float32)
        self.block_tables = self.meta[self._o_bt:].view(B, self.max_blocks)
        self.feed = self.meta[lay["feed"]:lay["feed"] + 1]
        self.tokens_host = torch.zeros(B, dtype=torch.int64, pin_memory=True)
        # Staged uploads and token read-backs of steps run ahead (``DecodeEngine.run_steps``): two
        # pinned copies of the metadata and of the tokens, used by alternate steps, so the host
        # never rewrites a buffer a queued copy may still read.
        self._meta_stage = [torch.zeros(lay["total"], dtype=torch.int32, pin_memory=True) for _ in range(2)]
        self._tok_stage = [torch.zeros(B, dtype=torch.int64, pin_memory=True) for _ in range(2)]
        self._stage_i = 0
        self._tok_event: list[torch.cuda.Event | None] = [None, None]
        self._host_sampling(0.0, -1, 1.0)
        self.upload_metadata()

        gemm_shapes = [(qkv_n, H), (H, self.Hq * self.D), (2 * self.I, H), (H, self.I), (self.Vl, H)]
        if self.moe:
            gemm_shapes.append((self.E, H))
        gemm_ws = max(N.lib().mvb_gemm_workspace_bytes(B, n, k, didx) for n, k in gemm_shapes)
        attn_ws = N.lib().mvb_paged_attention_workspace_bytes(B, self.Hq, self.D, didx)
        self.gemm_ws = torch.zeros(gemm_ws, dtype=torch.uint8, device=dev)
        self.attn_ws = torch.zeros(attn_ws, dtype=torch.uint8, device=dev)
        self.graph: torch.cuda.CUDAGraph | None = None
        self.graph_stream: torch.cuda.Stream | None = None
        eligible = (not self.gemma and not self.moe and B <= 64 and self.D == 128 and H % 64 == 0 and H <= 4096 and
                    self.I % 64 == 0 and not cfg.get("_rms_norm_plus_one"))
        if fused_layers and not eligible:
            raise ValueError("the fused layer kernel needs a dense model, batch <= 64, head dim 128, hidden <= 4096 "
                             "and a per-rank intermediate size that is a multiple of 64")
        self.fused = bool(fused_layers)
        if self.fused:
            lib = N.lib()
            self.layer_ws = torch.zeros(lib.mvb_decoder_layer_workspace_bytes(B, H, self.Hq * self.D, self.I, qkv_n,
                                                                              didx), dtype=torch.uint8, device=dev)
            self.layer_bar = torch.zeros(256, dtype=torch.uint8, device=dev)

    # ----------------------------------------------------------------- metadata
    def set_metadata(self, ids: list[int], positions: list[int], block_tables: list[list[int]], offset: int = 0,
                     ctx_lens: list[int] | None = None) -> None:
        """Fills the pinned host mirror for the rows given; the rest are padded rows that
        write into the pool's scratch block and attend to one token there."""
        n = len(ids)
        if n > self.B:
            raise ValueError(f"batch {n} exceeds the runner's max_batch {self.B}")
        m = self.meta_host
        B, mb = self.B, self.max_blocks
        m[:self._o_off + 2].zero_()
        m[0:n] = torch.tensor(ids, dtype=torch.int32)
        m[self._o_pos:self._o_pos + n] = torch.tensor(positions, dtype=torch.int32)
        ctx = ctx_lens if ctx_lens is not None else [p + 1 for p in positions]
        m[self._o_ctx:self._o_ctx + n] = torch.tensor(ctx, dtype=torch.int32)
        if n < B:
            m[self._o_ctx + n:self._o_ctx + B] = 1
        m[self._o_off:self._o_off + 2] = torch.tensor([offset], dtype=torch.int64).view(torch.int32)
        bt = m[self._o_bt:].view(B, mb)
        bt.fill_(self.kv.scratch_block)
        for i, t in enumerate(block_tables):
            if len(t) > mb:
                raise ValueError(f"sequence needs {len(t)} blocks > max_blocks {mb}")
            bt[i, :len(t)] = torch.tensor(t, dtype=torch.int32)

    def upload_metadata(self) -> None:
        self.meta.copy_(self.meta_host, non_blocking=True)

    def launch_staged(self, feed: bool) -> int:
        """Copies the host metadata into the next staging buffer (``feed`` set or not), uploads
        it and replays the step, then queues the read-back of the step's tokens into the matching
        token buffer.  Returns the buffer index for ``tokens_of``.  Nothing waits on the host."""
        i = self._stage_i
        self._stage_i ^= 1
        m = self._meta_stage[i]
        m.copy_(self.meta_host)
        m[self.meta_offsets["feed"]] = 1 if feed else 0
        self.meta.copy_(m, non_blocking=True)
        self.replay()
        self._tok_stage[i].copy_(self.tokens, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.dev))
        self._tok_event[i] = ev
        return i

    def tokens_of(self, i: int) -> torch.Tensor:
        """The tokens of the step launched by ``launch_staged`` into buffer ``i`` (waits for them)."""
        self._tok_event[i].synchronize()
        return self._tok_stage[i]

    def _host_sampling(self, temperature, top_k, top_p) -> None:
        lay, B, m = self.meta_offsets, self.B, self.meta_host
        m[lay["temp"]:lay["temp"] + B].view(torch.float32).copy_(
            torch.as_tensor(temperature, dtype=torch.float32).expand(B))
        m[lay["topk"]:lay["topk"] + B].copy_(torch.as_tensor(top_k, dtype=torch.int32).expand(B))
        m[lay["topp"]:lay["topp"] + B].view(torch.float32).copy_(torch.as_tensor(top_p, dtype=torch.float32).expand(B))

    def set_sampling(self, temperature, top_k, top_p, seed: int = 0) -> None:
        """Per-row (or scalar) sampling parameters; T == 0 rows decode greedily.  They sit in the
        step metadata (host mirror and device copy are both updated here)."""
        self._host_sampling(temperature, top_k, top_p)
        lay, B = self.meta_offsets, self.B
        self.meta[lay["temp"]:lay["topp"] + B].copy_(self.meta_host[lay["temp"]:lay["topp"] + B])
        if int(seed) != self.seed:
            self.seed = int(seed)
            self.graph = None  # the seed is a kernel argument: re-capture

    def set_probs_out(self, enabled: bool) -> None:
        """With ``enabled`` the step's sampler also writes each row's filtered, tempered
        probabilities to ``self.probs`` ``[B, V]`` fp32 (the distribution a parity-mode draw uses)."""
        want = bool(enabled)
        if want == (self.probs is not None):
            return
        self.probs = torch.zeros(self.B, self.V, dtype=torch.float32, device=self.dev) if want else None
        self.graph = None

    # ------------------------------------------------------------------- step
    def _gemm(self, y, x, w, epilogue=N.EPI_STORE, aux=None):
        """y = x @ w.T on the tcgen05 GEMM; with EPI_PARTIALS (y None) the result stays in the
        workspace as split-K partials for the next kernel to reduce."""
        lib = N.lib()
        B = self.B
        N.check(lib.mvb_gemm_bf16(N.ptr(y), 0 if y is None else y.stride(0), x.data_ptr(), x.stride(0),
                                  w.data_ptr(), w.stride(0), B,
                                  w.shape[0], w.shape[1], epilogue, N.ptr(aux), 0 if aux is None else aux.stride(0),
                                  self.gemm_ws.data_ptr(), self.gemm_ws.numel(), self._st), "gemm_bf16")

    def _qk(self, i) -> None:
        """QK-norm + RoPE + KV write of layer i from the q|k|v projection's split-K partials."""
        w, D = self.w, self.D
        cos, sin = self.layer_tables[i]
        N.check(N.lib().mvb_qk_norm_rope_kv_write_gemm(
            self.q.data_ptr(), self.kv.kv_cache.data_ptr(), self.gemm_ws.data_ptr(), self.H,
            w.qn[i].data_ptr() if w.qk_norm else None, w.kn[i].data_ptr() if w.qk_norm else None,
            cos.data_ptr(), sin.data_ptr(), cos.shape[0], self.pos.data_ptr(), self.block_tables.data_ptr(),
            self.max_blocks, self.B, self.Hq, self.Hkv, D, self.L, i, self.P, self.kv.block_size, self.eps,
            self.plus_one, self._st), "qk_norm_rope_kv_write_gemm")

    def _attention(self, i) -> None:
        """Paged decode attention of layer i (soft-capping and sliding window as configured)."""
        D = self.D
        N.check(N.lib().mvb_paged_attention_decode_ex(
            self.attn.data_ptr(), self.attn.stride(0), self.q.data_ptr(), self.Hq * D, self.kv.kv_cache.data_ptr(),
            self.block_tables.data_ptr(), self.max_blocks, self.ctx.data_ptr(), self.B, self.Hq, self.Hkv, D,
            self.L, i, self.P, self.kv.block_size, self.scale, self.softcap, self.windows[i],
            self.attn_ws.data_ptr(), self.attn_ws.numel(), self._st), "paged_attention_decode")

    def _add_norm(self, gemm_k, weight, post_weight=None) -> None:
        """residual += the preceding GEMM's output (Gemma: post-normalised first), xn = norm(residual)."""
        lib, B, H = N.lib(), self.B, self.H
        if post_weight is not None:
            N.check(lib.mvb_fused_norm_add_rmsnorm_gemm(self.xn.data_ptr(), self.residual.data_ptr(),
                                                        self.gemm_ws.data_ptr(), B, H, gemm_k,
                                                        post_weight.data_ptr(), weight.data_ptr(), self.eps,
                                                        self.plus_one, self._st), "fused_norm_add_rmsnorm_gemm")
        else:
            N.check(lib.mvb_fused_add_rmsnorm_gemm(self.xn.data_ptr(), self.residual.data_ptr(),
                                                   self.gemm_ws.data_ptr(), B, H, gemm_k, weight.data_ptr(),
                                                   self.eps, self.plus_one, self._st), "fused_add_rmsnorm_gemm")

    def _embed(self) -> None:
        """Token embedding (times sqrt(hidden) for Gemma) and the first layer's input norm."""
        lib, w, B, H = N.lib(), self.w, self.B, self.H
        N.check(lib.mvb_embedding(self.residual.data_ptr(), self.ids.data_ptr(), N.I32, w.embed.data_ptr(), B, H,
                                  self.V, self.embed_scale, N.BF16, self._st), "embedding")
        N.check(lib.mvb_rmsnorm(self.xn.data_ptr(), H, self.residual.data_ptr(), H, w.ln1[0].data_ptr(), B, H,
                                self.eps, self.plus_one, N.NORM_MODEL, N.BF16, self._st), "rmsnorm")

    def _logits_and_sample(self) -> None:
        """lm_head into the logits buffer, the final soft-capping (Gemma-2), sampling."""
        lib, B = N.lib(), self.B
        self._gemm(self.logits, self.xn, self.w.lm_head)
        if self.final_softcap:
            N.check(lib.mvb_softcap(self.logits.data_ptr(), B * self.V, self.final_softcap, N.BF16, self._st),
                    "softcap")
        N.check(lib.mvb_sample(self.tokens.data_ptr(), N.ptr(self.probs), self.logits.data_ptr(), B, self.V, self.V,
                               self.temperature.data_ptr(), self.top_k.data_ptr(), self.top_p.data_ptr(), self.seed,
                               0, self.offset.data_ptr(), N.BF16, self._st), "sample")

    def _layer_tail(self, i) -> None:
        """Layer i after its attention, and the next layer's q|k|v projection, QK-norm, RoPE and KV
        write: one fused launch (``mvb_decoder_layer_tail``)."""
        w, B, H, D = self.w, self.B, self.H, self.D
        nxt = i + 1 < self.L
        cos, sin = self.layer_tables[i + 1] if nxt else self.layer_tables[i]
        N.check(N.lib().mvb_decoder_layer_tail(
            self.attn.data_ptr(), self.attn.stride(0), w.wo[i].data_ptr(), w.ln2[i].data_ptr(), w.wgu[i].data_ptr(),
            w.wdown[i].data_ptr(), (w.ln1[i + 1] if nxt else w.final_norm).data_ptr(),
            w.wqkv[i + 1].data_ptr() if nxt else None,
            w.qn[i + 1].data_ptr() if nxt and w.qk_norm else None, w.kn[i + 1].data_ptr() if nxt and w.qk_norm else None,
            self.residual.data_ptr(), self.xn.data_ptr(), self.h.data_ptr(), self.q.data_ptr(),
            self.kv.kv_cache.data_ptr(), cos.data_ptr(), sin.data_ptr(), cos.shape[0], self.pos.data_ptr(),
            self.block_tables.data_ptr(), self.max_blocks, B, H, self.Hq, self.Hkv, D, self.I, self.L,
            i + 1 if nxt else 0, self.P, self.kv.block_size, self.eps, self.layer_ws.data_ptr(), self.layer_ws.numel(),
            self.layer_bar.data_ptr(), self._st), "decoder_layer_tail")

    def _forward_fused(self) -> None:
        """The dense step with fused layers: embedding, input norm, layer 0's q|k|v GEMM and
        QK-norm/RoPE/KV write, then per layer its attention and one fused launch for the rest (and
        the next layer's projection), lm_head and sampling: 2L + 6 launches."""
        self._st = N.stream_handle(self.dev)
        self._embed()
        self._gemm(None, self.xn, self.w.wqkv[0], N.EPI_PARTIALS)
        self._qk(0)
        for i in range(self.L):
            self._attention(i)
            self._layer_tail(i)
        self._logits_and_sample()

    def forward(self) -> None:
        """Launches one decode step on the current stream (metadata must be on the device)."""
        self._st = N.stream_handle(self.dev)
        N.check(N.lib().mvb_feed_ids(self.ids.data_ptr(), self.tokens.data_ptr(), self.feed.data_ptr(), self.B,
                                     self._st), "feed_ids")
        if self.tp.enabled:
            self._forward_tp()
            return
        if self.moe:
            self._forward_moe()
            return
        if self.fused:
            self._forward_fused()
            return
        lib, w, B, H = N.lib(), self.w, self.B, self.H
        self._st = N.stream_handle(self.dev)
        st = self._st
        g = self.gemma   # Gemma: post-norms of the attention and MLP outputs before each residual add
        self._embed()
        for i in range(self.L):
            if i > 0:   # residual += down_proj output (split-K partials), then input_layernorm
                self._add_norm(self.I, w.ln1[i], w.post_ff[i - 1] if g else None)
            self._gemm(None, self.xn, w.wqkv[i], N.EPI_PARTIALS)
            self._qk(i)
            self._attention(i)
            self._gemm(None, self.attn, w.wo[i], N.EPI_PARTIALS)
            if g:   # residual += post_attention_layernorm(o_proj), then pre_feedforward_layernorm
                self._add_norm(self.Hq * self.D, w.pre_ff[i], w.ln2[i])
            else:
                self._add_norm(self.Hq * self.D, w.ln2[i])
            self._gemm(None, self.xn, w.wgu[i], N.EPI_SWIGLU_PARTIALS)
            N.check(lib.mvb_gated_gemm(self.h.data_ptr(), self.h.stride(0), self.gemm_ws.data_ptr(), B, self.I, H,
                                       self.act, st), "gated_gemm")
            self._gemm(None, self.h, w.wdown[i], N.EPI_PARTIALS)
        self._add_norm(self.I, w.final_norm, w.post_ff[self.L - 1] if g else None)
        self._logits_and_sample()

    def _moe_mlp(self, i) -> None:
        """The sparse MoE block on ``self.xn`` into ``self.mlp_out`` (``qwen3_moe_model.py:39-65``):
        router GEMM, routing + dispatch order, gather, grouped gate/up (SwiGLU) and down GEMMs over
        the active experts, expert-ordered weighted combine.  Tensor parallel: every rank routes
        every row, computes its own experts only, and pushes its combined partial to the row's
        owner (``mvb_tp_moe_combine``, signal point ``point_down(i)``)."""
        lib, w, B, H, st = N.lib(), self.w, self.B, self.H, self._st
        if self.tp.enabled:
            self._gemm(self.router_logits, self.xn, w.router[i])
            N.check(lib.mvb_moe_route(self.router_logits.data_ptr(), B, self.E, self.K, self.norm_topk,
                                      self.topk_ids.data_ptr(), self.topk_w.data_ptr(), self.pair_row.data_ptr(),
                                      self.row_token.data_ptr(), self.expert_off.data_ptr(), self.active.data_ptr(),
                                      st), "moe_route")
            n = B * self.K
            N.check(lib.mvb_moe_gather(self.x_sorted.data_ptr(), self.xn.data_ptr(), H, self.row_token.data_ptr(), n,
                                       st), "moe_gather")
            for y, ldy, x, ldx, wt, nn, k, epi in (
                    (self.h_sorted, self.Im, self.x_sorted, H, w.egu[i], 2 * self.Im, H, N.EPI_SWIGLU),
                    (self.y_sorted, H, self.h_sorted, self.Im, w.edown[i], H, self.Im, N.EPI_STORE)):
                N.check(lib.mvb_moe_gemm_bf16_experts(y.data_ptr(), ldy, x.data_ptr(), ldx, wt.data_ptr(), nn, k,
                                                      self.E, self.e_first, self.e_local, n, B, epi,
                                                      self.expert_off.data_ptr(), self.active.data_ptr(), st),
                        "moe_gemm_experts")
            N.check(lib.mvb_tp_moe_combine(self.heap.comm, self.y_sorted.data_ptr(), self.topk_w.data_ptr(),
                                           self.topk_ids.data_ptr(), self.pair_row.data_ptr(), B, self.K, H,
                                           self.e_first, self.e_local, self.layout.recv_down, tpm.point_down(i), st),
                    "tp_moe_combine")
            return
        self._gemm(self.router_logits, self.xn, w.router[i])
        N.check(lib.mvb_moe_route(self.router_logits.data_ptr(), B, self.E, self.K, self.norm_topk,
                                  self.topk_ids.data_ptr(), self.topk_w.data_ptr(), self.pair_row.data_ptr(),
                                  self.row_token.data_ptr(), self.expert_off.data_ptr(), self.active.data_ptr(), st),
                "moe_route")
        n = B * self.K
        N.check(lib.mvb_moe_gather(self.x_sorted.data_ptr(), self.xn.data_ptr(), H, self.row_token.data_ptr(), n, st),
                "moe_gather")
        N.check(lib.mvb_moe_gemm_bf16(self.h_sorted.data_ptr(), self.Im, self.x_sorted.data_ptr(), H,
                                      w.egu[i].data_ptr(), 2 * self.Im, H, self.E, n, B, N.EPI_SWIGLU,
                                      self.expert_off.data_ptr(), self.active.data_ptr(), st), "moe_gemm gate_up")
        N.check(lib.mvb_moe_gemm_bf16(self.y_sorted.data_ptr(), H, self.h_sorted.data_ptr(), self.Im,
                                      w.edown[i].data_ptr(), H, self.Im, self.E, n, B, N.EPI_STORE,
                                      self.expert_off.data_ptr(), self.active.data_ptr(), st), "moe_gemm down")
        N.check(lib.mvb_moe_combine(self.mlp_out.data_ptr(), self.y_sorted.data_ptr(), self.topk_w.data_ptr(),
                                    self.topk_ids.data_ptr(), self.pair_row.data_ptr(), B, self.K, H, st),
                "moe_combine")

    def _forward_moe(self) -> None:
        """The step of a sparse-MoE model: the dense attention half as ``forward``, the MoE block
        in place of the MLP, and a plain residual add + RMSNorm after it."""
        lib, w, B, H, D = N.lib(), self.w, self.B, self.H, self.D
        self._st = N.stream_handle(self.dev)
        st, eps, bf = self._st, self.eps, N.BF16
        ws = self.gemm_ws.data_ptr()
        N.check(lib.mvb_embedding(self.residual.data_ptr(), self.ids.data_ptr(), N.I32, w.embed.data_ptr(), B, H,
                                  self.V, 1.0, bf, st), "embedding")
        N.check(lib.mvb_rmsnorm(self.xn.data_ptr(), H, self.residual.data_ptr(), H, w.ln1[0].data_ptr(), B, H, eps, 0,
                                N.NORM_MODEL, bf, st), "rmsnorm")
        for i in range(self.L):
            if i > 0:   # residual += MoE output, then input_layernorm
                N.check(lib.mvb_fused_add_rmsnorm(self.xn.data_ptr(), self.residual.data_ptr(), self.mlp_out.data_ptr(),
                                                  w.ln1[i].data_ptr(), B, H, eps, 0, N.NORM_MODEL, bf, st),
                        "fused_add_rmsnorm")
            self._gemm(None, self.xn, w.wqkv[i], N.EPI_PARTIALS)
            self._qk(i)
            self._attention(i)
            self._gemm(None, self.attn, w.wo[i], N.EPI_PARTIALS)
            N.check(lib.mvb_fused_add_rmsnorm_gemm(self.xn.data_ptr(), self.residual.data_ptr(), ws, B, H,
                                                   self.Hq * D, w.ln2[i].data_ptr(), eps, 0, st),
                    "fused_add_rmsnorm_gemm")
            self._moe_mlp(i)
        N.check(lib.mvb_fused_add_rmsnorm(self.xn.data_ptr(), self.residual.data_ptr(), self.mlp_out.data_ptr(),
                                          w.final_norm.data_ptr(), B, H, eps, 0, N.NORM_MODEL, bf, st),
                "fused_add_rmsnorm")
        self._gemm(self.logits, self.xn, w.lm_head)
        N.check(lib.mvb_sample(self.tokens.data_ptr(), N.ptr(self.probs), self.logits.data_ptr(), B, self.V, self.V,
                               self.temperature.data_ptr(), self.top_k.data_ptr(), self.top_p.data_ptr(), self.seed,
                               0, self.offset.data_ptr(), bf, st), "sample")

    def _tp_gemm(self, x, w, epilogue, out_offset=-1, ldy=0, wait=-1, signal=-1):
        N.check(N.lib().mvb_tp_gemm_bf16(self.heap.comm, x.data_ptr(), x.stride(0), w.data_ptr(), w.stride(0), self.B,
                                         w.shape[0], w.shape[1], epilogue, self.gemm_ws.data_ptr(),
                                         self.gemm_ws.numel(), out_offset, ldy, wait, signal, self._st),
                "tp_gemm_bf16")

    def _tp_add_norm(self, gemm_k, weight, recv, wait, signal, post=None):
        if post is not None:   # Gemma: the summed output is post-normalised before the residual add
            N.check(N.lib().mvb_tp_fused_norm_add_rmsnorm_gemm(
                self.heap.comm, self.residual.data_ptr(), self.B, self.H, gemm_k, post.data_ptr(), weight.data_ptr(),
                self.eps, self.plus_one, recv, wait, self.layout.xn, signal, self._st), "tp_fused_norm_add_rmsnorm_gemm")
            return
        N.check(N.lib().mvb_tp_fused_add_rmsnorm_gemm(self.heap.comm, self.residual.data_ptr(), self.B, self.H, gemm_k,
                                                      weight.data_ptr(), self.eps, self.plus_one, recv, wait,
                                                      self.layout.xn, signal, self._st), "tp_fused_add_rmsnorm_gemm")

    def _tp_layer_tail(self, i) -> None:
        """Tensor parallel: layer i after its attention and the next layer's projection as one
        launch (``mvb_tp_decoder_layer_tail``), the exchanges of the row-parallel o_proj and
        down_proj inside it (signal points 4i .. 4i + 3, as the per-kernel step uses them)."""
        w, B, H, D = self.w, self.B, self.H, self.D
        nxt = i + 1 < self.L
        cos, sin = self.layer_tables[i + 1] if nxt else self.layer_tables[i]
        N.check(N.lib().mvb_tp_decoder_layer_tail(
            self.heap.comm, i, self.attn.data_ptr(), self.attn.stride(0), w.wo[i].data_ptr(), w.ln2[i].data_ptr(),
            w.wgu[i].data_ptr(), w.wdown[i].data_ptr(), (w.ln1[i + 1] if nxt else w.final_norm).data_ptr(),
            w.wqkv[i + 1].data_ptr() if nxt else None,
            w.qn[i + 1].data_ptr() if nxt and w.qk_norm else None, w.kn[i + 1].data_ptr() if nxt and w.qk_norm else None,
            self.residual.data_ptr(), self.layout.xn, self.h.data_ptr(), self.q.data_ptr(), self.kv.kv_cache.data_ptr(),
            cos.data_ptr(), sin.data_ptr(), cos.shape[0], self.pos.data_ptr(), self.block_tables.data_ptr(),
            self.max_blocks, B, H, self.Hq, self.Hkv, D, self.I, self.L, i + 1 if nxt else 0, self.P,
            self.kv.block_size, self.eps, self.layout.recv_o, self.layout.recv_down, self.layer_ws.data_ptr(),
            self.layer_ws.numel(), self.layer_bar.data_ptr(), self._st), "tp_decoder_layer_tail")

    def _forward_tp(self) -> None:
        """The step on one rank of a tensor-parallel group (see tensor_parallel): same kernels,
        local head / feature counts, and the cross-GPU exchanges inside the row-parallel GEMMs,
        the add+norm kernels, the lm_head GEMM and one wait before sampling.  With fused layers,
        one launch per layer after its attention holds the layer's exchanges."""
        lib, w, B, H, D = N.lib(), self.w, self.B, self.H, self.D
        self._st = N.stream_handle(self.dev)
        st, eps, bf, lay = self._st, self.eps, N.BF16, self.layout
        comm = self.heap.comm
        ws = self.gemm_ws.data_ptr()
        N.check(lib.mvb_tp_begin_step(comm, st), "tp_begin_step")
        self._embed()
        if self.fused:
            self._tp_gemm(self.xn, w.wqkv[0], N.EPI_PARTIALS)
            self._qk(0)
            for i in range(self.L):
                self._attention(i)
                self._tp_layer_tail(i)   # the last one applies the final norm
        elif self.moe:
            self._tp_layers_moe()
        else:
            self._tp_layers()
        last = self.L - 1
        # vocab-parallel lm_head: this rank's columns into every rank's full logits
        self._tp_gemm(self.xn, w.lm_head, N.EPI_STORE, out_offset=lay.logits + self.tp.rank * self.Vl * 2,
                      ldy=self.V, wait=tpm.point_mlp_norm(last), signal=tpm.point_logits(self.L))
        N.check(lib.mvb_tp_wait(comm, tpm.point_logits(self.L), st), "tp_wait")
        if self.final_softcap:   # every rank soft-caps its copy of the gathered logits
            N.check(lib.mvb_softcap(self.logits.data_ptr(), B * self.V, self.final_softcap, N.BF16, st), "softcap")
        N.check(lib.mvb_sample(self.tokens.data_ptr(), N.ptr(self.probs), self.logits.data_ptr(), B, self.V, self.V,
                               self.temperature.data_ptr(), self.top_k.data_ptr(), self.top_p.data_ptr(), self.seed,
                               0, self.offset.data_ptr(), bf, st), "sample")

    def _tp_layers_moe(self) -> None:
        """Tensor-parallel attention and expert-parallel MoE blocks, through the final norm: the
        owners' add+norm sums one pushed partial per rank (a one-k-block plan, ``gemm_k`` 64)."""
        lib, w, D, st, lay = N.lib(), self.w, self.D, self._st, self.layout
        comm = self.heap.comm
        for i in range(self.L):
            if i > 0:
                self._tp_add_norm(64, w.ln1[i], lay.recv_down, tpm.point_down(i - 1), tpm.point_mlp_norm(i - 1))
            self._tp_gemm(self.xn, w.wqkv[i], N.EPI_PARTIALS, wait=-1 if i == 0 else tpm.point_mlp_norm(i - 1))
            self._qk(i)
            self._attention(i)
            self._tp_gemm(self.attn, w.wo[i], N.EPI_PARTIALS, out_offset=lay.recv_o, signal=tpm.point_o_proj(i))
            self._tp_add_norm(self.Hq * D, w.ln2[i], lay.recv_o, tpm.point_o_proj(i), tpm.point_attn_norm(i))
            N.check(lib.mvb_tp_wait(comm, tpm.point_attn_norm(i), st), "tp_wait")   # the router reads every row
            self._moe_mlp(i)
        last = self.L - 1
        self._tp_add_norm(64, w.final_norm, lay.recv_down, tpm.point_down(last), tpm.point_mlp_norm(last))

    def _tp_layers(self) -> None:
        """The per-kernel tensor-parallel layers, through the final norm."""
        lib, w, B, H, D = N.lib(), self.w, self.B, self.H, self.D
        st, lay = self._st, self.layout
        ws = self.gemm_ws.data_ptr()
        g = self.gemma   # Gemma: post-norms of the attention and MLP outputs before each residual add
        for i in range(self.L):
            if i > 0:
                self._tp_add_norm(self.I, w.ln1[i], lay.recv_down, tpm.point_down(i - 1), tpm.point_mlp_norm(i - 1),
                                  post=w.post_ff[i - 1] if g else None)
            self._tp_gemm(self.xn, w.wqkv[i], N.EPI_PARTIALS, wait=-1 if i == 0 else tpm.point_mlp_norm(i - 1))
            self._qk(i)
            self._attention(i)
            self._tp_gemm(self.attn, w.wo[i], N.EPI_PARTIALS, out_offset=lay.recv_o, signal=tpm.point_o_proj(i))
            self._tp_add_norm(self.Hq * D, w.pre_ff[i] if g else w.ln2[i], lay.recv_o, tpm.point_o_proj(i),
                              tpm.point_attn_norm(i), post=w.ln2[i] if g else None)
            self._tp_gemm(self.xn, w.wgu[i], N.EPI_SWIGLU_PARTIALS, wait=tpm.point_attn_norm(i))
            N.check(lib.mvb_gated_gemm(self.h.data_ptr(), self.h.stride(0), ws, B, self.I, H, self.act, st),
                    "gated_gemm")
            self._tp_gemm(self.h, w.wdown[i], N.EPI_PARTIALS, out_offset=lay.recv_down, signal=tpm.point_down(i))
        last = self.L - 1
        self._tp_add_norm(self.I, w.final_norm, lay.recv_down, tpm.point_down(last), tpm.point_mlp_norm(last),
                          post=w.post_ff[last] if g else None)

    def kernel_kinds(self) -> dict:
        """kind -> (launch(layer), launches per step, algorithmic bytes per launch, flops per launch)."""
        lib, w, B, H, D = N.lib(), self.w, self.B, self.H, self.D
        self._st = N.stream_handle(self.dev)
        st = self._st
        ctx = self.ctx.cpu().tolist()
        qkv_n = (self.Hq + 2 * self.Hkv) * D
        glob = [i for i in range(self.L) if not self.windows[i]]
        slid = [i for i in range(self.L) if self.windows[i]]

        def attn_kind(layers):   # launches over the given layers, bytes and flops of one launch
            wnd = self.windows[layers[0]]
            keys = sum(min(c, wnd) if wnd else c for c in ctx)
            return ((lambda i: self._attention(layers[i % len(layers)])), len(layers),
                    keys * self.Hkv * D * 2 * 2 + 2 * B * self.Hq * D * 2, 4 * keys * self.Hq * D)
        g = self.gemma

        def gemm_bytes(n, k, out_cols):
            return n * k * 2 + B * k * 2 + B * out_cols * 2

        def fadd(i):
            if g:
                self._add_norm(self.Hq * D, w.pre_ff[i], w.ln2[i])
            else:
                self._add_norm(self.Hq * D, w.ln2[i])

        def gated(i):
            N.check(lib.mvb_gated_gemm(self.h.data_ptr(), self.h.stride(0), self.gemm_ws.data_ptr(), B, self.I, H,
                                       self.act, st), "gated_gemm")

        def samp(i):
            N.check(lib.mvb_sample(self.tokens.data_ptr(), N.ptr(self.probs), self.logits.data_ptr(), B, self.V, self.V,
                                   self.temperature.data_ptr(), self.top_k.data_ptr(), self.top_p.data_ptr(),
                                   self.seed, 0, self.offset.data_ptr(), N.BF16, st), "sample")

        kinds = {}
        if glob:
            kinds["paged_attention_decode"] = attn_kind(glob)
        if slid:   # sliding-window layers: the newest `window` keys of each sequence
            kinds["paged_attention_decode_window"] = attn_kind(slid)
        kinds.update({
            "gemm_qkv": (lambda i: self._gemm(None, self.xn, w.wqkv[i], N.EPI_PARTIALS), self.L,
                         gemm_bytes(qkv_n, H, 0), 2 * B * qkv_n * H),
            "gemm_o_proj": (lambda i: self._gemm(None, self.attn, w.wo[i], N.EPI_PARTIALS), self.L,
                            gemm_bytes(H, self.Hq * D, 0), 2 * B * H * self.Hq * D),
            "gemm_gate_up": (lambda i: self._gemm(None, self.xn, w.wgu[i], N.EPI_SWIGLU_PARTIALS), self.L,
                             gemm_bytes(2 * self.I, H, 0), 2 * B * 2 * self.I * H),
            "swiglu_gemm": (gated, self.L, B * 2 * self.I * 4 + B * self.I * 2, 0),
            "gemm_down": (lambda i: self._gemm(None, self.h, w.wdown[i], N.EPI_PARTIALS), self.L,
                          gemm_bytes(H, self.I, 0), 2 * B * H * self.I),
            "gemm_lm_head": (lambda i: self._gemm(self.logits, self.xn, w.lm_head), 1,
                             gemm_bytes(self.Vl, H, self.Vl), 2 * B * self.Vl * H),
            "qk_norm_rope_kv_write": (self._qk, self.L, B * qkv_n * 2 + B * self.Hq * D * 2 + 2 * B * self.Hkv * D * 2,
                                      0),
            "fused_add_rmsnorm": (fadd, 2 * self.L, 5 * B * H * 2, 0),
            "sample": (samp, 1, B * self.V * 2, 0),
        })
        if self.final_softcap:
            kinds["softcap"] = (lambda i: N.check(lib.mvb_softcap(self.logits.data_ptr(), B * self.V,
                                                                  self.final_softcap, N.BF16, st), "softcap"),
                                1, 2 * B * self.V * 2, 0)
        if self.fused:   # the kinds the fused step launches
            tail_w = (H * self.Hq * D + 2 * self.I * H + H * self.I + qkv_n * H) * 2 + 3 * H * 2 + 2 * D * 2
            tail_act = (B * self.Hq * D + 4 * B * H + 2 * B * self.I + B * self.Hq * D) * 2 + 2 * B * self.Hkv * D * 2
            tail_flops = 2 * B * (H * self.Hq * D + 2 * self.I * H + H * self.I + qkv_n * H)
            keep = {k: kinds[k] for k in ("paged_attention_decode", "gemm_lm_head", "sample") if k in kinds}
            keep["gemm_qkv"] = (kinds["gemm_qkv"][0], 1, kinds["gemm_qkv"][2], kinds["gemm_qkv"][3])
            keep["qk_norm_rope_kv_write"] = (self._qk, 1, kinds["qk_norm_rope_kv_write"][2], 0)
            keep["decoder_layer_tail"] = (lambda i: self._layer_tail(i % max(self.L - 1, 1)), self.L, tail_w + tail_act,
                                          tail_flops)
            return keep
        return kinds

    def time_kernels(self, iters: int = 36) -> dict[str, dict]:
        """Average device time of each kernel kind: every launch bracketed by CUDA events on
        the launching stream, rotating over the layers (a working set far larger than L2)."""
        self._st = N.stream_handle(self.dev)
        stream = torch.cuda.current_stream(self.dev)
        out = {}
        for name, (fn, per_step, nbytes, flops) in self.kernel_kinds().items():
            fn(0)
            ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(iters)]
            torch.cuda.synchronize(self.dev)
            for it in range(iters):
                ev[it][0].record(stream)
                fn(it % self.L)
                ev[it][1].record(stream)
            torch.cuda.synchronize(self.dev)
            ms = sorted(a.elapsed_time(b) for a, b in ev)
            avg = sum(ms) / len(ms)
            out[name] = {"avg_ms": avg, "median_ms": ms[len(ms) // 2], "launches_per_step": per_step,
                         "bytes_per_launch": nbytes, "flops_per_launch": flops,
                         "gbs": nbytes / (avg * 1e-3) / 1e9}
        return out

    def algorithmic_step_bytes(self) -> int:
        """HBM bytes a decode step cannot avoid at the current context lengths: streamed weights,
        K and V of every attended token in every layer (a sliding-window layer attends to at most
        its window), and the new token's K and V."""
        ctx = self.ctx.cpu().tolist()
        per_layer = self.Hkv * self.D * 2 * 2
        attended = sum(sum(min(c, wnd) if wnd else c for c in ctx) for wnd in self.windows)
        return self.w.streamed_bytes() + attended * per_layer + self.B * self.L * per_layer

    def launches_per_step(self) -> int:
        """Kernels one step launches: the id feed, embedding, rmsnorm, 8 per layer (qkv,
        qk-norm/rope/kv, attention, o_proj, add+norm, gate_up, swiglu, down), an add+norm between
        layers, final add+norm, lm_head, sample."""
        return 1 + self._launches_after_feed()

    def _launches_after_feed(self) -> int:
        if self.moe:   # 11 per layer: qkv, qk, attention, o_proj, add+norm, router, route, gather, 2 GEMMs, combine
            # (tensor parallel: + a wait before each router, the step-counter kernel, the wait before sampling)
            return 2 + self.L * 11 + (self.L - 1) + 3 + (self.L + 2 if self.tp.enabled else 0)
        if self.fused:   # embedding, rmsnorm, qkv, qk, then attention + fused tail per layer, lm_head, sample
            # (tensor parallel: + the step-counter kernel and the wait before sampling)
            return 4 + 2 * self.L + 2 + (2 + (1 if self.final_softcap else 0) if self.tp.enabled else 0)
        if self.tp.enabled:   # + the step-counter kernel and the wait before sampling
            return 2 + self.L * 8 + (self.L - 1) + 3 + 2 + (1 if self.final_softcap else 0)
        return 2 + self.L * 8 + (self.L - 1) + 3 + (1 if self.final_softcap else 0)

    # ------------------------------------------------------------------ graphs
    def capture(self) -> None:
        """Records one full step in a CUDA graph (metadata and sampling buffers are read at replay)."""
        torch.cuda.synchronize(self.dev)
        s = torch.cuda.Stream(self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(s):
            self.forward()  # warm-up outside the graph: sets function attributes, loads modules
        s.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            self.forward()
        torch.cuda.synchronize(self.dev)
        self.graph, self.graph_stream = g, s

    def replay(self) -> None:
        if self.graph is None:
            self.capture()
        self.graph.replay()

    def step(self, use_graph: bool = True) -> None:
        """Metadata upload + one step on the current stream (no host sync)."""
        self.upload_metadata()
        if use_graph:
            self.replay()
        else:
            self.forward()

    def close(self) -> None:
        """Releases the graph, then the symmetric heap (tensor parallel)."""
        self.graph = None
        if self.heap is not None:
            torch.cuda.synchronize(self.dev)
            self.xn = self.logits = None
            self.heap.close()
            self.heap = None

    def fetch_tokens(self) -> torch.Tensor:
        self.tokens_host.copy_(self.tokens, non_blocking=True)
        torch.cuda.current_stream(self.dev).synchronize()
        return self.tokens_host
