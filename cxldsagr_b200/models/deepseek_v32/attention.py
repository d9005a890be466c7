"""One layer of DSA attention: projections -> indexer -> exact top-k -> KV
append / recall -> sparse MLA -> value expansion -> o_proj.

Reference pipeline: ``models/deepseek_v32/attention.py:276-425`` (runner) and
``models/deepseek_v32/projections.py:182-293`` (projections).  Differences of
the B200 design: the q_a / kv_a / indexer-wk linears run as one FP8 GEMM on
the quantised normed input, q_b and indexer wq_b as another; the KV record is
written by the projection epilogue straight into its pool row; the indexer
reads the resident FP8 key cache through TMA and the selection feeds the MLA
kernel without a host round trip in the resident (``hbm``) method.

Cache methods (``CacheConfig.method``):
* ``hbm``            resident main KV (logical row = physical row);
* ``serial_sparse``  finite HBM pool + pinned DRAM; exact recall after top-k;
* ``echo``           as serial_sparse, plus a prefetch of the subset of the
                     coming top-k that the coarse logit histogram proves, issued
                     on a copy stream while the exact top-k runs;
* ``dense_prefetch`` whole-history copy-engine DMA into the pool (one layer
                     ahead), then attention on resident rows.
"""

from __future__ import annotations

from contextlib import nullcontext

import torch

from ... import ops
from ...cache.indexer_cache import IndexerCache
from ...cache.sparse_token_cache import SparseTokenCache, WorkingSetTooLarge
from .weights import AttentionWeights


class LayerState:
    """Per-(session, layer) state: main KV view + resident FP8 indexer keys."""

    def __init__(self, kv: SparseTokenCache, index: IndexerCache):
        self.kv = kv
        self.index = index
        self.dense = None       # dense_prefetch: staged [rows, 576] history of this layer for the current chunk
        self.last_rows = None   # physical rows of the chunk's new records

    @property
    def cache(self):
        return self.kv


class AttentionRunner:
    """Stateless w.r.t. requests: every call gets the session's :class:`LayerState`."""

    def __init__(self, cfg, weights: AttentionWeights, *, method: str = "hbm"):
        self.cfg = cfg
        self.w = weights
        self.method = method
        # Rows per indexer + top-k round (0: the whole chunk at once).  A round's
        # FP32 logits (rows x context x 4 B) stay in L2 between the two kernels.
        # Off by default: on B200 at 64K context and 2048-token chunks the
        # whole chunk measured 548.3 ms per prefill against 559.3 ms with
        # 296-row rounds and 574.5 ms with 148-row rounds (smaller launches
        # cost more than the L2 residency saves).
        self.select_rows = 0
        # CUDA, methods other than echo (whose predictor reads the full logits):
        # indexer + top-k as one fused selection (ops.indexer_select).
        self.fused_select = True
        # Chunks of at most this many query rows prefetch the output-side
        # weights into L2 during selection + MLA.  Off (0): measured on B200,
        # 1-token extend at 64K, 1.034-1.042 ms with it and 1.039 ms without.
        self.prefetch_rows = 0
        self._side = None
        self._prefetch_done = None
        self.last_indices = None
        self.head_scale = cfg.index_n_heads ** -0.5 * cfg.index_head_dim ** -0.5
        (self.qa0, self.qa_n), (self.kv0, self.kv_n), (self.ik0, self.ik_n) = weights.spans_a
        (self.qb0, self.qb_n), (self.iq0, self.iq_n) = weights.spans_b

    # ------------------------------------------------------------- projection
    def project(self, state: LayerState, normed, quantized, pos: int, positions, freqs, scope=None,
                comm=None, rows=None):
        """Projections of one chunk.

        ``normed`` / ``quantized`` are this rank's query rows [r0, r1) of the
        chunk (all rows when not sequence parallel).  Under sequence
        parallelism ``comm.ag_linear`` all-gathers the chunk's input inside the
        q_a / kv_a / indexer-k GEMM (one fused kernel on the peer-memory
        backend); the latent KV record and the indexer key are produced for
        every row (the KV cache is replicated), the query path only for local rows.
        """
        scope = scope or (lambda _name: nullcontext())
        cfg, w = self.cfg, self.w
        T_loc = normed.shape[0]
        H, nope, rope, L = cfg.n_heads, cfg.qk_nope_head_dim, cfg.qk_rope_head_dim, cfg.kv_lora_rank
        r0, r1 = rows if rows is not None else (0, T_loc)
        with scope("fused_a_gemm"):
            if comm is not None and comm.world > 1:
                fp8 = w.fused_a.scales is not None
                a = comm.ag_linear(w.fused_a, normed, quantized if fp8 else None, positions.shape[0])
            else:
                a = w.fused_a(normed, quantized=quantized)
        T = a.shape[0]
        qa = a[r0:r1, self.qa0:self.qa0 + self.qa_n]
        kv = a[:, self.kv0:self.kv0 + self.kv_n]
        ik = a[:, self.ik0:self.ik0 + self.ik_n]
        # KV record straight into its cache row (every row of the chunk).
        with scope("kv_record"):
            with scope("slots"):
                dst = state.kv.destination_rows(T)
            packed = state.kv.packed_rows(T)  # FP8 caches: the 656-byte records of this chunk
            k_rows, s_rows = state.index.rows(pos, T)
            with scope("finish"):
                # KV records and the indexer keys of the chunk: one launch.
                ops.kv_finish_index_k(kv, L, rope, w.kv_norm, cfg.norm_eps, freqs, positions, state.kv.records, dst,
                                      ik, w.index_norm_w, w.index_norm_b, cfg.norm_eps, k_rows, s_rows,
                                      packed=packed)
            with scope("host_write"):
                state.kv.finish_append(dst, packed)
            state.last_rows = dst
            if state.dense is not None:
                # The staged history plus this chunk's records (logical row = staged row).
                state.dense[pos:pos + T] = state.kv.records[dst]
        if T_loc == 0:
            return None, None, None
        q_pos = positions[r0:r1]
        with scope("q_norm"):
            qa_normed, _, qr8, qrs = ops.norm_quant(qa, None, w.q_norm, cfg.norm_eps, want_out=w.fused_b.scales is None)
        with scope("fused_b_gemm"):
            b = w.fused_b(qa_normed, quantized=(qr8, qrs))
        q_proj = torch.empty((T_loc, H, cfg.qk_head_dim), dtype=torch.bfloat16, device=normed.device)
        with scope("absorb"):
            ops.mla_absorb(b, H, nope, rope, w.wk_b_t, q_proj)
        with scope("index_weights_f32"):
            w_raw = ops.linear_split(normed, w.index_head_split) if normed.is_cuda else ops.linear_f32(normed, w.index_head)
        iq = b[:, self.iq0:self.iq0 + self.iq_n]
        with scope("q_rope_index_q"):
            # MLA query RoPE and the indexer query (RoPE + FP8 + head weights): one launch.
            q_idx, weights = ops.mla_q_rope_index_q(b, H, nope, rope, freqs, q_pos, q_proj, L, iq,
                                                    cfg.index_n_heads, cfg.index_head_dim, rope, w_raw,
                                                    self.head_scale)
        return q_proj, q_idx, weights

    # ---------------------------------------------------------------- forward
    def forward(self, state: LayerState, normed, quantized, pos: int, positions, freqs, *, scope=None,
                logits_buf=None, comm=None, rows=None):
        """One chunk of attention; returns o_proj output for this rank's query rows."""
        scope = scope or (lambda _name: nullcontext())
        cfg = self.cfg
        T_loc = normed.shape[0]
        T = positions.shape[0]
        r0, r1 = rows if rows is not None else (0, T_loc)
        end = pos + T
        cache = state.kv
        with cache.operation():
            with scope("attention_projection"):
                q_proj, q_idx, weights = self.project(state, normed, quantized, pos, positions, freqs, scope,
                                                      comm=comm, rows=(r0, r1))
            if T_loc == 0:
                return torch.empty((0, cfg.dim), dtype=torch.bfloat16, device=normed.device)
            self._prefetch_done = None
            if normed.is_cuda and T_loc <= self.prefetch_rows:
                # Decode sizes: selection and sparse MLA below are latency-bound and
                # leave HBM idle, so the output projection's weights (and the value
                # expansion's) are pulled into L2 meanwhile, on a side stream that
                # the output joins (the prefetch kernel ends only when its bulk
                # prefetches have, so in stream order it would hold up the selection).
                cur = torch.cuda.current_stream(normed.device)
                if self._side is None:
                    self._side = torch.cuda.Stream(device=normed.device)
                self._side.wait_stream(cur)
                with torch.cuda.stream(self._side):
                    ops.l2_prefetch(self.w.wv_b)
                    ops.l2_prefetch(self.w.wo.weight)
                self._prefetch_done = torch.cuda.Event()
                self._prefetch_done.record(self._side)
            qpos = pos + r0
            keys, kscales = state.index.visible(end)
            if comm is not None and comm.world > 1 and getattr(comm.ctx, "cp_indexer", False) and \
                    self.method != "echo":
                # Context-parallel selection: every rank scores all of the chunk's
                # queries against its key shard, the (score, id) lists are merged.
                with scope("indexer_cp"):
                    ids = self._cp_select(comm, q_idx, weights, keys, kscales, pos, end, T, r0, r1)
                self.last_indices = ids
                with scope("sparse_mla"):
                    if state.dense is not None:
                        attn = ops.sparse_mla(q_proj, state.dense, ids, cfg.attention_scale,
                                              value_dim=cfg.kv_lora_rank,
                                              splits=ops.mla_splits(q_proj.shape[0], ids.shape[1]))
                    else:
                        attn = self._consume(cache, q_proj, ids)
                return self._output(attn, T_loc, scope)
            if normed.is_cuda and self.fused_select and self.method != "echo":
                # Fused exact selection: no full logits in HBM (sampled threshold,
                # candidate lists, candidate top-k; flagged rows redone in full).
                with scope("indexer_select"):
                    lb = logits_buf if (logits_buf is not None and logits_buf.shape[0] >= T_loc
                                        and logits_buf.shape[1] >= end) else None
                    _, ids = ops.indexer_select(q_idx, keys, weights, kscales, qpos, cfg.index_topk,
                                                logits_buf=lb, order="index")
                self.last_indices = ids
                with scope("sparse_mla"):
                    if state.dense is not None:
                        attn = ops.sparse_mla(q_proj, state.dense, ids, cfg.attention_scale,
                                              value_dim=cfg.kv_lora_rank,
                                              splits=ops.mla_splits(q_proj.shape[0], ids.shape[1]))
                    else:
                        attn = self._consume(cache, q_proj, ids)
                return self._output(attn, T_loc, scope)
            rounds = self._select_rounds(T_loc, end, normed.is_cuda)
            if rounds is not None:
                ids = self._select_in_rounds(rounds, q_idx, keys, weights, kscales, logits_buf, qpos, end, scope)
                values = None
                self.last_indices = ids
                with scope("sparse_mla"):
                    if state.dense is not None:
                        attn = ops.sparse_mla(q_proj, state.dense, ids, cfg.attention_scale,
                                              value_dim=cfg.kv_lora_rank)
                    else:
                        attn = self._consume(cache, q_proj, ids)
                return self._output(attn, T_loc, scope)
            with scope("indexer"):
                if logits_buf is not None and logits_buf.shape[0] >= T_loc and logits_buf.shape[1] >= end:
                    logits = logits_buf[:T_loc]
                else:
                    logits = torch.empty((T_loc, max(4, (end + 3) // 4 * 4)), dtype=torch.float32,
                                         device=normed.device)
                if logits.is_cuda:
                    ops.lib().indexer_logits(q_idx, keys, weights, kscales, logits, qpos)
                else:
                    logits = ops.indexer_logits(q_idx, keys, weights, kscales, qpos)
            if self.method == "echo" and cache.offload and pos > 0:
                with scope("indexer_prefetch"):
                    self._predictive_prefetch(state, logits, pos, end)
            with scope("exact_topk"):
                # The selection in ascending index order: the kernel skips its final
                # sort, and attention only needs the set in a deterministic order.
                values, ids = ops.exact_topk(logits, cfg.index_topk, causal_start=qpos, n=end, order="index")
            if self.method == "echo" and cache.offload:
                with scope("prefetch_hint"):
                    self._update_hints(state, logits, values, pos, end)
            self.last_indices = ids
            with scope("sparse_mla"):
                if state.dense is not None:
                    attn = ops.sparse_mla(q_proj, state.dense, ids, cfg.attention_scale, value_dim=cfg.kv_lora_rank,
                                          splits=ops.mla_splits(q_proj.shape[0], ids.shape[1]))
                else:
                    attn = self._consume(cache, q_proj, ids)
        return self._output(attn, T_loc, scope)

    def _cp_select(self, comm, q_idx, weights, keys, kscales, pos: int, end: int, T: int, r0: int, r1: int):
        """Exact top-k of this rank's query rows [r0, r1) with the indexer split by keys.

        The chunk's indexer queries and head weights are all-gathered; rank r
        scores all T queries against keys [k0, k1) of the visible ``end`` keys
        (``parallel.cp_indexer``), every rank's (score, id) lists are
        all-gathered and merged.  The selection equals the single-device one,
        ties included; ids come in descending-score order."""
        from ...parallel import cp_indexer as cp

        ctx = comm.ctx
        H, D = q_idx.shape[1], q_idx.shape[2]
        q_all = comm.gather_rows(q_idx.reshape(q_idx.shape[0], H * D), T).reshape(T, H, D)
        w_all = comm.gather_rows(weights.contiguous(), T)
        k0, k1 = cp.key_shard(end, ctx.world, ctx.rank)
        values, ids = cp.cp_exact_topk(ctx, q_all, keys[k0:k1], w_all, kscales[k0:k1], k0, pos, self.cfg.index_topk)
        return ids[r0:r1].contiguous()

    def _output(self, attn, T_loc, scope):
        if self._prefetch_done is not None:
            torch.cuda.current_stream(attn.device).wait_event(self._prefetch_done)
            self._prefetch_done = None
        with scope("attention_output"):
            with scope("expand"):
                v = ops.mla_expand(attn, self.w.wv_b)
            with scope("o_proj"):
                return self.w.wo(v.reshape(T_loc, -1))

    def _select_rounds(self, T_loc: int, end: int, cuda: bool):
        """Row rounds for the indexer + top-k, or None to run the chunk at once.

        Rounds apply on CUDA outside the echo method (whose predictor reads the
        whole chunk's logits), when the chunk is larger than one round and one
        round's logits fit comfortably in L2 (<= 96 MB)."""
        n = self.select_rows
        if not cuda or n <= 0 or self.method == "echo" or T_loc <= n or n * end * 4 > 96 * 2**20:
            return None
        k = -(-T_loc // n)              # rounds
        rows = -(-T_loc // k)           # equal rounds
        return [(s0, min(T_loc, s0 + rows)) for s0 in range(0, T_loc, rows)]

    def _select_in_rounds(self, rounds, q_idx, keys, weights, kscales, logits_buf, qpos, end, scope):
        cfg = self.cfg
        count = min(cfg.index_topk, end)
        T_loc = q_idx.shape[0]
        values = torch.empty((T_loc, count), dtype=torch.float32, device=q_idx.device)
        ids = torch.empty((T_loc, count), dtype=torch.int32, device=q_idx.device)
        n = max(r1 - r0 for r0, r1 in rounds)
        cols = max(4, (end + 3) // 4 * 4)
        if logits_buf is not None and logits_buf.shape[0] >= n and logits_buf.shape[1] >= end:
            buf = logits_buf
        else:
            buf = torch.empty((n, cols), dtype=torch.float32, device=q_idx.device)
        for r0, r1 in rounds:
            lg = buf[:r1 - r0]
            with scope("indexer"):
                ops.lib().indexer_logits(q_idx[r0:r1], keys, weights[r0:r1], kscales, lg, qpos + r0)
            with scope("exact_topk"):
                ops.exact_topk(lg, cfg.index_topk, causal_start=qpos + r0, n=end, order="index",
                               out=(values[r0:r1], ids[r0:r1]))
        return ids

    def _consume(self, cache, q, ids):
        if not cache.offload:
            return ops.sparse_mla(q, cache.records, ids, self.cfg.attention_scale, value_dim=self.cfg.kv_lora_rank,
                                  splits=ops.mla_splits(q.shape[0], ids.shape[1]))
        try:
            physical = cache.ensure(ids)
        except WorkingSetTooLarge:
            if len(q) == 1:
                raise ValueError("the pool must fit one query's exact selection") from None
            cache.stats.capacity_splits += 1
            mid = len(q) // 2
            return torch.cat((self._consume(cache, q[:mid], ids[:mid]), self._consume(cache, q[mid:], ids[mid:])))
        return ops.sparse_mla(q, cache.records, physical, self.cfg.attention_scale, value_dim=self.cfg.kv_lora_rank,
                              splits=ops.mla_splits(q.shape[0], ids.shape[1]))

    # ------------------------------------------------------------ echo method
    def _predictive_prefetch(self, state, logits, pos, end):
        """Prefetch the provable part of the coming top-k (coarse histogram threshold).

        For each query, bucket ``logit - offset[0]`` into 256 monotone bins; the
        bin holding the k-th element is the threshold; history tokens in strictly
        higher bins are certainly selected and are recalled now (reference
        predictor: operators/deepseek_v32/indexer/csrc/echo_logits.cuh:500-584).
        Budget: min(8192, P - Q) records.
        """
        k = self.cfg.index_topk
        cache = state.kv
        hist_end = min(pos, cache.length)
        if hist_end <= k:
            return
        budget = min(8192, cache.slots - logits.shape[0])
        if budget <= 0:
            return
        if logits.is_cuda and getattr(cache, "native", False):
            # Device predictor + device recall: no host synchronisation.
            pred = state.index.pred_ids(hist_end)
            ops.lib().echo_predict(logits, logits.shape[0], hist_end, state.index.offset, k, pred)
            cache.prefetch(pred, limit=budget)
            return
        rows = logits[:, :hist_end] - state.index.offset[0]
        key = _order_bins(rows)
        counts = torch.zeros((rows.shape[0], 257), dtype=torch.int64, device=rows.device)
        counts.scatter_add_(1, key.long(), torch.ones_like(key, dtype=torch.int64))
        above = counts.flip(1).cumsum(1).flip(1)  # elements in bins >= b
        thr = (above[:, 1:] > k).sum(1)            # first bin with <= k elements above it
        pred = key > thr[:, None]
        cand = torch.nonzero(pred.any(0)).flatten()
        if cand.numel():
            cache.prefetch(cand, limit=budget)

    def _update_hints(self, state, logits, values, pos, end):
        off = state.index.offset
        if logits.is_cuda:
            ops.lib().echo_hint(logits, logits.shape[0], end, off)  # one kernel, no host sync
        else:
            off[0] = ops.reference.prefetch_hint(logits[:, :end])
        if logits.shape[0] == 1 and end >= 32768:
            # kth score = the smallest selected one (the selection is index-ordered)
            off[1] = ops.reference.decode_hint(off[1], values[0].min())


def _order_bins(x: torch.Tensor) -> torch.Tensor:
    """256 monotone bins of FP16-ordered values (upper 8 bits of an order-preserving key)."""
    h = x.clamp(-65504, 65504).half().view(torch.int16).int()
    key = torch.where(h < 0, (~h) & 0xFFFF, h | 0x8000)
    return (key >> 8).clamp(0, 255) + 1
