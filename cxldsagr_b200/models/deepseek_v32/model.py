"""DeepSeek-V3.2 model: embedding -> DSA blocks -> final norm -> last-token LM head.

Reference: ``models/deepseek_v32/model.py:63-980`` (model + transactional
forward), ``layers.py:215-344`` (block), ``layers.py:54-212`` (MLP / MoE).

One forward call is one cache *step* for every layer: ``begin_step`` on all
layer caches, the tokens run through the blocks in chunks of ``chunk_size``
(prefill) and the step is committed only when every chunk succeeded;
otherwise every layer rolls back and all cleanup errors are collected in one
``BaseExceptionGroup`` (reference: ``model.py:778-814``).  A *transient*
forward (candidate tokens of a GR request) writes KV only to the pool's GPU
tail rows and is always discarded afterwards.

The extend step can be captured once into a CUDA graph (:meth:`capture_extend`)
and replayed per request, like the reference's full extend graph
(``models/deepseek_v32/execution/extend_graph.py``).
"""

from __future__ import annotations

import functools
from contextlib import nullcontext
from dataclasses import dataclass

import torch

from ... import ops
from ...cache.indexer_cache import IndexerCache
from ...cache.sparse_token_cache import SparseTokenCache
from ...cache.sparse_token_pool import SharedSparseTokenPool
from ...config import CacheConfig, ModelConfig
from ...parallel.comm import make_comm
from ...parallel.groups import ParallelContext, shard_range, single
from .attention import AttentionRunner, LayerState
from .replay import ReplayLayout
from .weights import MLPWeights, MoEWeights, load_attention, load_mlp, load_moe


class DenseMLP:
    """SwiGLU MLP.  Under sequence parallelism the weights are column/row sharded:
    gather the chunk (AG -> gate_up GEMM), SiLU*up, then the row-parallel down
    GEMM whose partial sums are reduce-scattered back to the row owners."""

    def __init__(self, w: MLPWeights, comm=None, sharded: bool = False):
        self.w = w
        self.comm = comm
        self.sharded = sharded

    def __call__(self, normed, quantized, scope=None, total: int | None = None):
        scope = scope or (lambda _n: nullcontext())
        tp = self.sharded and self.comm is not None and self.comm.world > 1
        with scope("gate_up_gemm"):
            if tp:
                fp8 = self.w.gate_up.scales is not None
                packed = self.comm.ag_linear(self.w.gate_up, normed, quantized if fp8 else None, total)
            else:
                packed = self.w.gate_up(normed, quantized=quantized)
        with scope("silu_mul_quant"):
            h, q, s_t = ops.silu_mul_quant(packed)
        with scope("down_gemm"):
            if tp:
                return self.comm.linear_rs(self.w.down, h, (q, s_t) if q is not None else None)
            return self.w.down(h, quantized=(q, s_t))


class MoE:
    """Routed experts (sigmoid group-limited top-k) plus the shared expert.

    Token rows are routed on the rank that holds them, dispatched to the
    expert owners (all-to-all under expert parallelism), run through the
    owner's expert GEMMs, sent back and combined per token in a fixed
    (token, k) slot order, so the sum is deterministic.
    """

    def __init__(self, cfg: ModelConfig, w: MoEWeights, comm=None, workspace: dict | None = None):
        self.cfg, self.w = cfg, w
        self.comm = comm
        self.shared = DenseMLP(w.shared) if w.shared is not None else None
        # Grouped-layout workspaces, shared by every MoE layer of the model (layers run one
        # after another) and bucketed by row count (powers of two) so memory stays bounded.
        self._layouts = workspace if workspace is not None else {}

    def _layout(self, rows: int, device):
        bucket = max(128, 1 << max(0, rows - 1).bit_length())
        key = (bucket, self.w.experts.start, len(self.w.experts), str(device))
        lay = self._layouts.get(key)
        if lay is None:
            lay = ops.MoELayout(bucket, self.w.experts.start, len(self.w.experts), self.cfg.dim, device)
            self._layouts[key] = lay
        return lay

    def _grouped(self, ids, q, s_t, topk: int):
        """Local experts over device-built grouped layout: gate_up -> SiLU*up (+FP8 quant) -> down."""
        w = self.w
        lay = self._layout(ids.numel(), q.device).build(ids, q, s_t, topk)
        gu = ops.fp8_gemm_grouped(lay.a, lay.a_s, w.w_gate_up, w.s_gate_up, lay.block_expert)
        _, hq, hs = ops.silu_mul_quant(gu)
        return ops.fp8_gemm_grouped(hq, hs, w.w_down, w.s_down, lay.block_expert), lay

    def _gpu(self, normed, quantized, scope, total):
        cfg, w = self.cfg, self.w
        T, K = normed.shape[0], cfg.num_experts_per_tok
        with scope("moe_gate"):
            if T:
                logits = ops.linear_split(normed, w.gate_split)
                ids, weights = ops.moe_route(logits, w.bias, cfg, split=True)
            else:
                ids = torch.empty((0, K), dtype=torch.int32, device=normed.device)
                weights = torch.empty((0, K), dtype=torch.float32, device=normed.device)
        q, s_t = quantized
        world = 1 if self.comm is None else self.comm.world
        if world == 1:
            with scope("moe_experts"):
                y, lay = self._grouped(ids, q, s_t, K)
            with scope("moe_combine"):
                out = ops.moe_combine(y, lay.positions, weights, T)
        elif hasattr(self.comm, "ep_ready") and self.comm.ep_ready(cfg.n_routed_experts, cfg.dim, K, total):
            def experts(a, a_s, block_expert, y_out):
                gu = ops.fp8_gemm_grouped(a, a_s, w.w_gate_up, w.s_gate_up, block_expert)
                _, hq, hs = ops.silu_mul_quant(gu)
                ops.fp8_gemm_grouped(hq, hs, w.w_down, w.s_down, block_expert, out=y_out)

            with scope("moe_ep_fused"):
                out = self.comm.moe_ep(ids, q, s_t, weights, experts)
        else:
            flat = ids.reshape(-1).long()
            per = cfg.n_routed_experts // world
            dest = flat // per
            order = torch.argsort(dest * cfg.n_routed_experts + flat, stable=True)
            token = order // K
            with scope("moe_dispatch"):
                rrows, rscales, rexp, sc, rc = self.comm.dispatch(q[token], s_t.t()[token].contiguous(), dest[order],
                                                                  flat[order])
            with scope("moe_experts"):
                y, lay = self._grouped(rexp.int(), rrows.contiguous(), rscales.t().contiguous(), 1)
                y_rows = y[lay.positions.long()]
            with scope("moe_combine"):
                back = self.comm.combine(y_rows, sc, rc)
                slots = torch.empty((T * K, cfg.dim), dtype=torch.bfloat16, device=normed.device)
                slots[order] = back
                out = (slots.view(T, K, cfg.dim).float() * weights.view(T, K, 1)).sum(1).bfloat16()
        if self.shared is not None:
            with scope("shared_expert"):
                out = (out.float() + self.shared(normed, quantized).float()).bfloat16()
        return out

    def _experts(self, x, s_rows, experts):
        """Run local experts over rows grouped by expert id; returns bf16 [N, D]."""
        cfg, w = self.cfg, self.w
        I = cfg.moe_intermediate_size
        out = torch.zeros((x.shape[0], cfg.dim), dtype=torch.bfloat16, device=x.device)
        if x.shape[0] == 0:
            return out
        local = experts.long() - w.experts.start
        order = torch.argsort(local, stable=True)
        counts = torch.bincount(local, minlength=len(w.experts)).tolist()
        start = 0
        for j, n in enumerate(counts):
            if n == 0:
                continue
            sel = order[start:start + n]
            start += n
            if w.s_gate_up is not None:
                q, s_t = x[sel], s_rows[sel].t().contiguous()
                packed = ops.fp8_gemm(q, s_t, w.w_gate_up[j], w.s_gate_up[j])
                _, hq, hs = ops.silu_mul_quant(packed)
                y = ops.fp8_gemm(hq, hs, w.w_down[j], w.s_down[j])
            else:
                packed = ops.linear(x[sel], w.w_gate_up[j])
                h = ops.silu_mul(packed[:, :I], packed[:, I:])
                y = ops.linear(h, w.w_down[j])
            out[sel] = y.to(torch.bfloat16)
        return out

    def __call__(self, normed, quantized, scope=None, total: int | None = None):
        cfg, w = self.cfg, self.w
        scope = scope or (lambda _n: nullcontext())
        if normed.is_cuda and w.s_gate_up is not None and w.gate_split is not None:
            return self._gpu(normed, quantized, scope, normed.shape[0] if total is None else total)
        T, K = normed.shape[0], cfg.num_experts_per_tok
        with scope("moe_gate"):
            ids, weights = ops.route_experts(normed, w.gate, w.bias, cfg)
        fp8 = w.s_gate_up is not None
        flat = ids.reshape(-1).long()
        world = 1 if self.comm is None else self.comm.world
        per = cfg.n_routed_experts // world if world > 1 else cfg.n_routed_experts
        dest = flat // per if world > 1 else torch.zeros_like(flat)
        order = torch.argsort(dest * cfg.n_routed_experts + flat, stable=True)   # by owner, then expert
        token = order // K
        if fp8:
            q, s_t = quantized
            rows, s_rows = q[token], s_t.t()[token].contiguous()
        else:
            rows, s_rows = normed[token], None
        with scope("moe_dispatch"):
            if world > 1:
                rrows, rscales, rexp, sc, rc = self.comm.dispatch(rows, s_rows, dest[order], flat[order])
            else:
                rrows, rscales, rexp = rows, s_rows, flat[order]
        with scope("moe_experts"):
            y = self._experts(rrows, rscales, rexp)
        with scope("moe_combine"):
            back = self.comm.combine(y, sc, rc) if world > 1 else y
            slots = torch.empty((T * K, cfg.dim), dtype=torch.bfloat16, device=normed.device)
            slots[order] = back
            out = (slots.view(T, K, cfg.dim).float() * weights.view(T, K, 1).float()).sum(1)
        if self.shared is not None:
            with scope("shared_expert"):
                out += self.shared(normed, quantized).float()
        return out.bfloat16()


class Block:
    def __init__(self, cfg: ModelConfig, layer: int, attention: AttentionRunner, mlp, post_norm, comm=None):
        self.cfg, self.layer = cfg, layer
        self.attention = attention
        self.mlp = mlp
        self.post_norm = post_norm
        self.comm = comm

    def forward(self, state, hidden, residual, pos, positions, freqs, *, scope=None, logits_buf=None, rows=None):
        """``hidden``/``residual`` hold this rank's rows ``rows=(r0, r1)`` of the chunk."""
        cfg = self.cfg
        scope = scope or (lambda _n: nullcontext())
        total = positions.shape[0]
        with scope("input_residual_norm"):
            normed, summed, q8, s8 = ops.norm_quant(hidden, residual, self.attention.w.input_norm, cfg.norm_eps)
        attn = self.attention.forward(state, normed, (q8, s8), pos, positions, freqs, scope=scope,
                                      logits_buf=logits_buf, comm=self.comm, rows=rows)
        with scope("post_attention_residual_norm"):
            normed2, out_res, q2, s2 = ops.norm_quant(summed, attn, self.post_norm, cfg.norm_eps)
        if isinstance(self.mlp, MoE):
            with scope("moe"):
                out = self.mlp(normed2, (q2, s2), scope, total=total)
        else:
            with scope("dense_mlp"):
                out = self.mlp(normed2, (q2, s2), scope, total=total)
        return out, out_res


class ModelSession:
    """One request history: per-layer KV views (resident or pool-backed) + indexer keys.

    ``length`` is the committed history; a failed step poisons nothing but
    the session's open step (rolled back); a session whose rollback failed is
    marked ``failed`` and cannot execute again.
    """

    def __init__(self, model: "DeepSeekV32Model", capacity: int):
        cc, width = model.cache_cfg, model.cfg.qk_head_dim
        self.model = model
        self.capacity = capacity
        # One pool session per device pool (layer placement); pool_session is the first.
        self.pool_sessions = [pool.allocate_session(capacity) for pool in model.pools] if cc.offload else []
        self.pool_session = self.pool_sessions[0] if self.pool_sessions else None
        self.layers: list[LayerState] = []
        for i in range(len(model.layer_ids)):
            dev = model.placement[i]
            if cc.offload:
                g, local = model.block_pool[i]
                kv = self.pool_sessions[g].layer(local)
            else:
                kv = SparseTokenCache(capacity, width, device=dev, candidate_slots=cc.candidate_tokens,
                                      kv_format=cc.kv_format, latent_dim=model.cfg.kv_lora_rank)
            index = IndexerCache(capacity + cc.candidate_tokens, model.cfg.index_head_dim, device=dev)
            self.layers.append(LayerState(kv, index))
        self.length = 0
        self.failed = False
        self.released = False

    @property
    def caches(self):
        return [layer.kv for layer in self.layers]

    def reset(self):
        for layer in self.layers:
            layer.kv.reset()
            layer.index.offset.zero_()
            layer.index.truncate(0)
        self.length = 0
        self.failed = False

    def truncate(self, length: int):
        for layer in self.layers:
            layer.kv.truncate(length)
            layer.index.truncate(length)
        self.length = length

    def bind_serving(self, lifecycle):
        """Guard this session's KV caches: mutation only inside the lifecycle's operation on this session."""
        check = functools.partial(lifecycle.check_active, self)
        for layer in self.layers:
            layer.kv.access_check = check

    def release(self):
        if self.released:
            return
        for ps in self.pool_sessions:
            ps.release()
        self.layers.clear()
        self.released = True

    def nbytes(self) -> dict:
        """Bytes owned by this session alone (shared pool rows are not counted)."""
        hbm = sum(layer.index.nbytes() for layer in self.layers)
        if self.pool_session is None:
            hbm += sum(layer.kv.records.numel() * layer.kv.records.element_size() for layer in self.layers)
        else:
            hbm += sum(ps.session_bytes().get("hbm", 0) for ps in self.pool_sessions)
        return {"hbm": hbm, "dram": 0}


@dataclass
class ForwardResult:
    logits: torch.Tensor      # fp32 [1, vocab] of the last token
    start: int
    length: int
    hidden: torch.Tensor | None = None  # final-normed bf16 [rows of the last chunk, dim] when requested


class DeepSeekV32Model:
    """A contiguous range of DeepSeek-V3.2 layers with embedding, final norm and LM head.

    ``source`` provides checkpoint tensors (:class:`CheckpointReader` or
    :class:`StateDictSource`).  ``cache`` chooses the KV method and sizes;
    offload methods share one :class:`SharedSparseTokenPool` across layers.
    """

    def __init__(self, cfg: ModelConfig, source, *, device="cuda", cache: CacheConfig | None = None,
                 layers=None, pool: SharedSparseTokenPool | None = None, scope=None,
                 allocate_default_session: bool = True, replay: bool = False, allocate_pool: bool = True,
                 parallel: ParallelContext | None = None, devices=None, reserve_gib: float = 8.0):
        """``devices``: place the layers over several devices of this process
        (contiguous runs by weight bytes, see :mod:`...parallel.placement`);
        the embedding lives on the first, final norm and LM head on the last."""
        self.cfg = cfg
        self.device = torch.device(devices[0] if devices else device)
        self.cache_cfg = cache or CacheConfig(capacity=4096)
        self.layer_ids = list(range(cfg.num_hidden_layers) if layers is None else layers)
        self.scope = scope
        self.par = parallel or single(self.device)
        if devices and len(devices) > 1:
            from ...parallel.placement import device_budgets, layer_weight_bytes, plan_layer_devices

            if self.par.world > 1:
                raise ValueError("layer placement runs in one process; it does not combine with a process group")
            devs = [torch.device(d) for d in devices]
            sizes = [layer_weight_bytes(cfg, layer, fp8=cfg.weight_dtype == "fp8") for layer in self.layer_ids]
            edge = cfg.vocab_size * cfg.dim * 2
            self.placement = plan_layer_devices(sizes, devs,
                                                device_budgets(devs, int(reserve_gib * 2**30), (edge, edge)))
        else:
            self.placement = [self.device] * len(self.layer_ids)
        self.head_device = self.placement[-1] if self.placement else self.device
        # Device pools: one per distinct device, holding that device's blocks in order.
        self.pool_devices = list(dict.fromkeys(self.placement)) or [self.device]
        self.block_pool = []
        for dv in self.placement:
            g = self.pool_devices.index(dv)
            self.block_pool.append((g, sum(1 for x in self.block_pool if x[0] == g)))
        has_moe = any(cfg.is_moe_layer(layer) for layer in self.layer_ids)
        self.comm = make_comm(self.par, max_rows=self.cache_cfg.chunk_size,
                              moe=(cfg.n_routed_experts, cfg.dim, cfg.num_experts_per_tok) if has_moe else None)
        # Replay: physical blocks are copies of checkpoint layers 0,1,2 repeated; blocks
        # >= 3 take clones of their source block's inputs (see replay.ReplayLayout).
        self.replay_layout = ReplayLayout(tuple(self.layer_ids)) if replay else None
        cc = self.cache_cfg
        dev = self.device
        hd = self.head_device
        # One request across ranks (world > 1): the embedding table and the LM
        # head are split by vocabulary rows, rank r keeping rows vocab_rows.
        self.vocab_parallel = self.par.world > 1 and getattr(self.par, "vocab_parallel", True)
        V = cfg.vocab_size
        self.vocab_rows = shard_range(V, self.par.world, self.par.rank) if self.vocab_parallel else (0, V)
        v0, v1 = self.vocab_rows

        def vocab_shard(name, device, dtype):
            full = source.get_tensor(name)
            return (full[v0:v1] if self.vocab_parallel else full).to(device, dtype).contiguous()

        self.embed_table = vocab_shard("model.embed_tokens.weight", dev, torch.bfloat16)
        self.final_norm = source.get_tensor("model.norm.weight").to(hd, torch.float32).contiguous()
        self.lm_head = vocab_shard("lm_head.weight", hd, torch.bfloat16)
        self._freqs = {d: ops.reference.rotary_frequencies(cfg, device=d) for d in self.pool_devices}
        self.freqs = self._freqs[self.pool_devices[0]]
        if len(self.pool_devices) > 1 and (cc.method == "dense_prefetch" or pool is not None or replay):
            raise ValueError("layer placement supports the hbm, serial_sparse and echo methods with own pools")
        self.pools: list[SharedSparseTokenPool] = []
        self.pool = None
        self.session = None
        if pool is not None:
            self.attach_pool(pool)
        elif cc.offload and allocate_pool:
            self._build_pools()
        self.blocks: list[Block] = []
        par, comm = self.par, self.comm
        self._moe_workspace: dict = {}
        for i, layer in enumerate(self.layer_ids):
            dev = self.placement[i]
            attn_w = load_attention(source, cfg, layer, device=dev)
            runner = AttentionRunner(cfg, attn_w, method=cc.method)
            if cfg.is_moe_layer(layer):
                experts = par.expert_range(cfg.n_routed_experts)
                mlp = MoE(cfg, load_moe(source, cfg, layer, device=dev, experts=experts), comm, self._moe_workspace)
            else:
                mw = load_mlp(source, cfg, f"model.layers.{layer}.mlp", device=dev, shard=(par.rank, par.world))
                mlp = DenseMLP(mw, comm, sharded=par.world > 1)
            post = source.get_tensor(f"model.layers.{layer}.post_attention_layernorm.weight").to(dev, torch.float32)
            self.blocks.append(Block(cfg, layer, runner, mlp, post.contiguous(), comm))
        self.dense_staging = None
        self._build_staging()
        self._logits_buf = {}
        self.last_hidden = None
        self.poisoned = False
        self.session = self.new_session(cc.capacity) if allocate_default_session else None

    # ------------------------------------------------------------- sessions
    def _build_pools(self):
        cc = self.cache_cfg
        P = cc.pool_tokens or min(cc.capacity, 65536)
        host = cc.host_tokens or cc.capacity
        if len(self.pool_devices) == 1:
            self.attach_pool(self.make_pool(host, P))
            return
        hp = (host + 63) // 64 * 64
        self.pools = [SharedSparseTokenPool(hp, self.cfg.qk_head_dim, sum(1 for x in self.block_pool if x[0] == g), P,
                                            device=d, candidate_slots=cc.candidate_tokens, kv_format=cc.kv_format,
                                            latent_dim=self.cfg.kv_lora_rank)
                      for g, d in enumerate(self.pool_devices)]
        self.pool = self.pools[0]

    def _build_staging(self):
        cc = self.cache_cfg
        if cc.method == "dense_prefetch":
            from ...cache.staging import DoubleBufferStaging

            self.dense_staging = DoubleBufferStaging(cc.capacity + cc.candidate_tokens, self.cfg.qk_head_dim,
                                                     device=self.device, fp8_records=cc.kv_format == "fp8",
                                                     latent_dim=self.cfg.kv_lora_rank)

    def set_cache_method(self, method: str, **overrides):
        """Switch to another cache method with an independent, empty cache.

        Reference: ``models/deepseek_v32/model.py:458-479``.  Every session of
        this model is released and the model's own pools are closed; new pools
        (offload methods) or staging buffers (``dense_prefetch``) are built
        from the cache config with ``method`` and ``overrides`` (for example
        ``pool_tokens``), and a new default session is opened.  Weights stay.
        """
        from dataclasses import replace

        if method not in ("hbm", "echo", "serial_sparse", "dense_prefetch"):
            raise ValueError("unsupported DeepSeek cache method")
        cc = replace(self.cache_cfg, method=method, **overrides)
        if method == "dense_prefetch" and (cc.pool_tokens or min(cc.capacity, 65536)) < cc.capacity:
            raise ValueError("dense prefetch requires P >= session capacity")
        if method == "dense_prefetch" and len(self.pool_devices) > 1:
            raise ValueError("layer placement supports the hbm, serial_sparse and echo methods with own pools")
        if self.session is not None:
            self.session.release()
            self.session = None
        for pool in self.pools:
            pool.close()
        self.pools, self.pool, self.dense_staging = [], None, None
        self.cache_cfg = cc
        for block in self.blocks:
            block.attention.method = method
        if cc.offload:
            self._build_pools()
        self._build_staging()
        self.session = self.new_session(cc.capacity)

    def snapshot_prefix(self, *, session: ModelSession | None = None) -> dict:
        """Snapshot a session's committed prefix (pool rows and maps, indexer lengths and hints).

        Reference: ``models/deepseek_v32/model.py:945-962``.  Resident (``hbm``)
        records keep their prefix untouched by later steps, so only lengths are
        recorded for them; offload pools are snapshotted whole (the pool must be
        quiescent).  ``restore_prefix`` rewinds the session to this point.
        """
        session = session or self.session
        if session.failed or session.released:
            raise RuntimeError("the session cannot be snapshotted")
        return {"schema": "cxld-prefix-v1", "model": id(self), "session": id(session),
                "method": self.cache_cfg.method, "length": session.length,
                "pools": [pool.snapshot() for pool in self.pools] if session.pool_session is not None else [],
                "index": [layer.index.snapshot() for layer in session.layers]}

    def restore_prefix(self, state: dict, *, session: ModelSession | None = None):
        session = session or self.session
        if (state.get("schema") != "cxld-prefix-v1" or state["model"] != id(self) or state["session"] != id(session)
                or state["method"] != self.cache_cfg.method or len(state["index"]) != len(session.layers)):
            raise ValueError("prefix snapshot does not match this model's cache")
        for pool, snap in zip(self.pools, state["pools"]):
            pool.restore(snap)
        for layer, idx in zip(session.layers, state["index"]):
            if session.pool_session is None:
                layer.kv.truncate(state["length"])
            layer.index.restore(idx)
        session.length = state["length"]

    def make_pool(self, host_tokens: int, pool_tokens: int) -> SharedSparseTokenPool:
        """A shared sparse-token pool for this model's layers (host rows rounded to 64-token pages)."""
        host = (host_tokens + 63) // 64 * 64
        return SharedSparseTokenPool(host, self.cfg.qk_head_dim, len(self.layer_ids), pool_tokens,
                                     device=self.device, candidate_slots=self.cache_cfg.candidate_tokens,
                                     kv_format=self.cache_cfg.kv_format, latent_dim=self.cfg.kv_lora_rank)

    def attach_pool(self, pool: SharedSparseTokenPool | None):
        if pool is not None and pool.num_layers != len(self.layer_ids):
            raise ValueError("the pool must have one layer per model block")
        if pool is not None and len(self.pool_devices) > 1:
            raise ValueError("a placed model builds one pool per device itself")
        self.pool = pool
        self.pools = [pool] if pool is not None else []

    def new_session(self, capacity: int | None = None) -> ModelSession:
        return ModelSession(self, capacity or self.cache_cfg.capacity)

    def release_session(self, session: ModelSession):
        session.release()

    @property
    def length(self) -> int:
        return self.session.length

    # -------------------------------------------------------------- helpers
    @property
    def caches(self):
        return self.session.caches

    def _scope(self):
        return self.scope or (lambda _n: nullcontext())

    def _ensure_logits_buf(self, rows, cols, device=None):
        device = device or self.device
        if not device.type == "cuda":
            return None
        cols = (cols + 3) // 4 * 4
        buf = self._logits_buf.get(device)
        if buf is None or buf.shape[0] < rows or buf.shape[1] < cols:
            cap_cols = max(cols, (self.cache_cfg.capacity + self.cache_cfg.candidate_tokens + 3) // 4 * 4)
            buf = torch.empty((max(rows, self.cache_cfg.chunk_size), cap_cols), dtype=torch.float32, device=device)
            self._logits_buf[device] = buf
        return buf

    # ------------------------------------------------------------- forward
    def _body(self, session: ModelSession, ids: torch.Tensor, start: int, chunk: int, want_hidden: bool = False):
        cfg = self.cfg
        scope = self._scope()
        T = ids.numel()
        par = self.par
        out_h, out_r, rows = None, None, (0, 0)
        for c0 in range(0, T, chunk):
            c1 = min(T, c0 + chunk)
            pos = start + c0
            positions = ops.arange_cached(pos, start + c1, device=self.device, dtype=torch.float32)
            pos_on = {self.device: positions}
            rows = par.token_range(c1 - c0)
            with scope("embedding"):
                if self.vocab_parallel:
                    # Every rank embeds the whole chunk from its vocabulary rows
                    # (zeros elsewhere); the sum lands on each row's owner.
                    partial = ops.embed(ids[c0:c1], self.embed_table, row0=self.vocab_rows[0],
                                        vocab_total=cfg.vocab_size)
                    hidden = self.comm.reduce_rows(partial)
                else:
                    hidden = ops.embed(ids[c0 + rows[0]:c0 + rows[1]], self.embed_table)
            residual = None
            n_rows = max(rows[1] - rows[0], 1)
            logits_buf = self._ensure_logits_buf(n_rows, start + c1)
            replay = self.replay_layout.begin_chunk() if self.replay_layout is not None else None
            dense = self.dense_staging is not None and session.pool_session is not None
            nxt = self._stage_history(session, 0, pos) if dense else None
            for i, (block, state) in enumerate(zip(self.blocks, session.layers)):
                if replay is not None:
                    with scope("replay_input_copy"):
                        hidden, residual = replay.for_layer(i, hidden, residual)
                cur = None
                if dense:
                    cur = nxt
                    with scope("dense_history_wait"):
                        cur.wait_ready()
                    state.dense = self.dense_staging.buffers[cur.index]
                    if i + 1 < len(self.blocks):  # next layer's history streams in meanwhile
                        nxt = self._stage_history(session, i + 1, pos)
                dv = self.placement[i]
                try:
                    if dv != hidden.device:  # layer placement: hand the rows to the next device
                        with scope("hidden_transfer"):
                            hidden = hidden.to(dv, non_blocking=True)
                            residual = residual.to(dv, non_blocking=True) if residual is not None else None
                    if dv not in pos_on:
                        pos_on[dv] = positions.to(dv)
                    lb = logits_buf if dv == self.device else self._ensure_logits_buf(n_rows, start + c1, dv)
                    with (torch.cuda.device(dv) if dv.type == "cuda" else nullcontext()):
                        hidden, residual = block.forward(state, hidden, residual, pos, pos_on[dv], self._freqs[dv],
                                                         scope=scope, logits_buf=lb, rows=rows)
                finally:
                    if cur is not None:
                        state.dense = None
                        cur.release()
            out_h, out_r = hidden, residual
        hd = self.head_device
        with scope("final_norm_lm_head"), (torch.cuda.device(hd) if hd.type == "cuda" else nullcontext()):
            n_last = c1 - c0
            owner = next(r for r in range(par.world) if par.world == 1 or
                         shard_range(n_last, par.world, r)[0] <= n_last - 1 < shard_range(n_last, par.world, r)[1])
            keep = slice(None) if want_hidden else slice(-1, None)
            normed = None
            if out_h.shape[0]:
                normed, _ = ops.residual_rms_norm(out_h[keep], out_r[keep], self.final_norm, cfg.norm_eps)
            head = (lambda x: ops.linear(x, self.lm_head).float()) if hd.type != "cuda" else self._lm_head
            if self.vocab_parallel:
                # The owner's last row goes to every rank; each computes the
                # logits of its vocabulary rows, then the shards are gathered.
                last = normed[-1:].contiguous() if par.rank == owner else torch.empty(
                    (1, cfg.dim), dtype=torch.bfloat16, device=hd)
                last = self.comm.broadcast(last, owner)
                logits = self.comm.gather_cols(head(last).contiguous(), cfg.vocab_size)
            else:
                logits = torch.empty((1, self.lm_head.shape[0]), dtype=torch.float32, device=hd)
                if par.rank == owner:
                    logits = head(normed[-1:])
                if par.world > 1:
                    logits = self.comm.broadcast(logits.contiguous(), owner)
            if par.world > 1 and want_hidden:
                local = normed if normed is not None else torch.empty((0, cfg.dim), dtype=torch.bfloat16,
                                                                     device=self.device)
                normed = self.comm.gather_rows(local, n_last)
        self.last_hidden = normed if want_hidden else None
        return logits

    def _stage_history(self, session, layer: int, rows: int):
        """Copy-engine DMA of layer ``layer``'s committed history [0, rows) from pinned host pages."""
        lease = self.dense_staging.lease()
        ps = session.pool_session
        host = self.pool.layers[layer].host
        runs = list(ps.host_runs(0, rows)) if rows else []
        return lease.prefetch_runs(host, runs, rows,
                                   before=lambda: self.pool.wait_host(ps, layer))

    def _lm_head(self, last):
        out = torch.empty((last.shape[0], self.lm_head.shape[0]), dtype=torch.float32, device=self.head_device)
        V, D = self.lm_head.shape
        ops.lib().bf16_gemm(last.contiguous(), 0, D, 0, self.lm_head, 0, D, 0, out, 0, V, 0, last.shape[0], V, D, 1)
        return out

    def forward(self, ids, *, session: ModelSession | None = None, transient: bool = False,
                chunk_size: int | None = None, commit: bool = True, return_hidden: bool = False):
        """Run ``ids`` after the session's committed history; returns last-token logits.

        ``transient``: candidate tokens (GR); their KV lives only in the GPU
        tail rows and is discarded (history length unchanged).
        """
        if self.poisoned:
            raise RuntimeError("model is poisoned after a failed cleanup")
        session = session or self.session
        if session.failed or session.released:
            raise RuntimeError("session cannot execute after a failure or release")
        ids = ids.to(self.device).reshape(-1)
        T = ids.numel()
        if T == 0:
            raise ValueError("empty token batch")
        start = session.length
        caches = session.caches
        for c in caches:
            (c.begin_transient if transient else c.begin_step)(T)
        chunk = chunk_size or self.cache_cfg.chunk_size
        if transient and any(c.offload for c in caches):
            chunk = T  # candidate rows are one batch
        try:
            logits = self._body(session, ids, start, chunk, want_hidden=return_hidden)
        except BaseException as primary:
            errors = []
            for c in caches:
                try:
                    c.rollback()
                except BaseException as exc:  # noqa: BLE001 - keep every cleanup failure
                    errors.append(exc)
            if errors:
                session.failed = True
                raise BaseExceptionGroup("forward and cache rollback failed", [primary, *errors]) from None
            raise
        if transient:
            for c in caches:
                c.discard_transient()
        elif commit:
            for c in caches:
                c.commit()
            for layer in session.layers:
                layer.index.commit(start + T)
            session.length = start + T
        return ForwardResult(logits, start, T, self.last_hidden)

    prefill = forward

    def extend(self, ids, **kw):
        return self.forward(ids, **kw)

    def candidate(self, ids, *, session: ModelSession | None = None):
        return self.forward(ids, session=session, transient=True)

    def truncate(self, length: int, *, session: ModelSession | None = None):
        (session or self.session).truncate(length)

    def clear_residency(self, *, session: ModelSession | None = None, rows_per_layer=None, seed: int = 0):
        """Drop the HBM copies of a session's offloaded history (host copies and indexer keys stay):
        the next steps recall every selected row from DRAM.

        ``rows_per_layer`` (one count per layer, in model layer order) drops
        only that many randomly chosen history rows of each layer instead of
        all of them, so a following extend recalls at most that many rows per
        layer; it pins the DRAM traffic of an extend to a given recall count."""
        session = session or self.session
        if session.pool_session is None or not self.pools:
            return
        gen = torch.Generator().manual_seed(seed)
        first = 0
        for pool, ps in zip(self.pools, session.pool_sessions):
            pool.drain()
            ids = ps.global_ids()
            for layer in range(pool.num_layers):
                drop = ids
                if rows_per_layer is not None:
                    hist = ids[: session.length]  # logical order: the committed history comes first
                    count = min(int(rows_per_layer[first + layer]), hist.numel())
                    pick = torch.randperm(hist.numel(), generator=gen)[:count].to(ids.device)
                    drop = hist[pick]
                pool.release_ids(layer, drop)
            first += pool.num_layers

    def reset(self, *, session: ModelSession | None = None):
        (session or self.session).reset()

    # --------------------------------------------------------- CUDA graph
    def capture_extend(self, T: int, *, warmup: int = 2, session: ModelSession | None = None) -> "ExtendGraph":
        """Capture a T-token extend at the session's history length into a CUDA graph."""
        return ExtendGraph(self, T, warmup=warmup, session=session)


class ExtendGraph:
    """One CUDA graph for a whole T-token extend step.

    Each replay re-opens the cache step on the host (cheap bookkeeping), copies
    the token ids into the static input and launches the graph; the caller
    commits with :meth:`commit` or discards with :meth:`rollback`.  Offload
    methods (serial_sparse, echo) are captured too: their pool metadata,
    predictor, recall and host write-back run on the device with no host
    decision inside the step, so every replay acts on the pool state of its
    own time.  dense_prefetch is captured with its staging stream: the
    whole-layer history copies from pinned host pages (one per contiguous
    run, fixed at the captured history length) become copy nodes of the graph
    ordered after the compute that last read their buffer.
    """

    def __init__(self, model: DeepSeekV32Model, T: int, *, warmup: int = 2, session: ModelSession | None = None):
        if len(model.pool_devices) > 1:
            raise ValueError("a model placed over several devices runs its extend eagerly")
        comm = getattr(model, "comm", None)
        if comm is not None and getattr(comm, "moe", None) is not None and comm.world > 1:
            # Its dispatch / combine number their calls on the host, which a replay would repeat.
            raise ValueError("the expert-parallel exchange runs its extend eagerly")
        self.model, self.T = model, T
        self.session = session or model.session
        self.start = self.session.length
        dev = model.device
        self.static_ids = torch.zeros(T, dtype=torch.int64, device=dev)
        model._ensure_logits_buf(T, self.start + T)
        stream = torch.cuda.Stream(device=dev)
        stream.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(stream):
            for _ in range(warmup):
                model.forward(self.static_ids, session=self.session, commit=False)
                self._rewind()
        torch.cuda.current_stream(dev).wait_stream(stream)
        pool = model.pool if self.session.pool_session is not None else None
        if pool is not None:
            pool.drain()   # no host-write ticket from before the capture is waited on inside it
        self.graph = torch.cuda.CUDAGraph()
        for c in self.session.caches:
            c.begin_step(T)
        from ...ops.native import launch_count

        n0 = launch_count()
        with torch.cuda.graph(self.graph, stream=stream):
            self.static_logits = model._body(self.session, self.static_ids, self.start, T)
            if pool is not None:
                pool.join_writes()
        if pool is not None:
            pool.end_capture()
        if getattr(model, "dense_staging", None) is not None:
            model.dense_staging.end_capture()
        self.launches_per_replay = launch_count() - n0
        model._graph_launches = self.launches_per_replay
        self._rewind()

    def _rewind(self):
        for c in self.session.caches:
            c._step_end = None
            if c.offload and max(c.written, c.length) > self.start:
                # Unmap the step's rows from the pool (their slots become free).
                top = max(c.written, c.length)
                ids = c.logical_to_global(torch.arange(self.start, top, device=c.device))
                c._pool.release_ids(c.layer_id, ids)
            c.written = c.length = self.start
        self.session.length = self.start

    def replay(self, ids: torch.Tensor):
        if self.session.length != self.start:
            raise RuntimeError("extend graph was captured at another history length")
        self.static_ids.copy_(ids.reshape(-1), non_blocking=True)
        for c in self.session.caches:
            c.begin_step(self.T)
            c.written = self.start + self.T
        self.graph.replay()
        return self.static_logits

    def commit(self):
        for c in self.session.caches:
            c.commit()
        for layer in self.session.layers:
            layer.index.commit(self.start + self.T)
        self.session.length = self.start + self.T

    def rollback(self):
        self._rewind()
