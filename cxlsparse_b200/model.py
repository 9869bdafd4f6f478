"""NSA-1B-shaped extend model around the selected-block transport.

The per-layer structure follows ``cxl_recsys/models/nsa/model.py:440-492,
592-827``: RMSNorm -> q/k/v/g projections -> RoPE -> compressed summaries
(ops.py:62-70) -> compressed branch + top-n -> selected transport with the
window branch and gate mix -> o_proj -> RMSNorm -> SwiGLU FFN. Projections and
the FFN are plain cuBLAS GEMMs through torch (out of scope for new kernels);
every attention branch, the planner and the backing-pool IO run in
``libcxlsparse_b200.so``.

Weights are random N(0, 0.02) (norm weights 1) with a fixed seed: no
checkpoint is needed to measure the path. ``prefill`` pushes a user's history
through the same layers in chunks, writing each layer's history KV into the
pinned backing pool (the reference's persistent KV write,
model.py:659-688); ``extend`` runs one GR candidate suffix over that history
without appending to it.
"""

import math
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

from . import _lib, ops
from .mempool import HiSparseCache, MemoryPool
from .segments import SegmentLayout
from .transport import GRSelectedTransport


@dataclass
class NSAConfig:
    layers: int = 16
    hidden: int = 2048
    q_heads: int = 32
    kv_heads: int = 2
    head_dim: int = 64
    ffn: int = 5632
    vocab: int = 32000
    rms_eps: float = 1e-6
    rope_theta: float = 10000.0
    block_size: int = 64
    block_counts: int = 16
    window: int = 512
    hot: int = 256
    # Compressed branch. "mean": the reference's summaries (mean of each
    # selection block, models/nsa/ops.py:62-70). "mlp": the NSA
    # paper's geometry (Yuan et al. 2025): a key/value per window of cmp_block tokens at stride
    # cmp_stride from a per-layer MLP with intra-window position encoding,
    # selection scores aggregated over the overlapping windows.
    compression: str = "mean"
    cmp_block: int = 32
    cmp_stride: int = 16
    cmp_hidden: int = 256
    forced_blocks: bool = False  # block 0 and the two local blocks always selected

    @property
    def groups(self):
        return self.q_heads // self.kv_heads

    @property
    def windows(self):
        """(window, stride) of the compressed keys."""
        if self.compression == "mean":
            return self.block_size, self.block_size
        return self.cmp_block, self.cmp_stride

    @classmethod
    def baseline(cls, **overrides):
        """The NSA paper's parameters (the serving benchmark's geometry): compression 32 / stride 16 with an MLP,
        selection block 64, top-16 including block 0 and 2 local blocks,
        window 512."""
        values = dict(compression="mlp", cmp_block=32, cmp_stride=16, forced_blocks=True)
        values.update(overrides)
        return cls(**values)


@dataclass
class UserState:
    row: int
    length: int = 0
    pages: list = field(default_factory=list)        # [layer][head] -> page list
    summaries: list = field(default_factory=list)    # [layer] -> [C, H, 128] bf16
    tails: list = field(default_factory=list)        # [layer] -> [<BS, H, 128]
    windows: list = field(default_factory=list)      # [layer] -> [<=W-1, H, 128]


def rms_norm(hidden, weight, eps):
    value = hidden.float()
    normalized = value * torch.rsqrt(value.square().mean(-1, keepdim=True) + eps)
    return normalized.to(hidden.dtype) * weight


def rotary(query, key, positions, inv_freq):
    frequency = positions.float()[:, None] * inv_freq[None, :]
    phase = torch.cat((frequency, frequency), -1)
    cosine = phase.cos().to(query.dtype)[:, None, :]
    sine = phase.sin().to(query.dtype)[:, None, :]

    def rotate(value):
        left, right = value.chunk(2, -1)
        return value * cosine + torch.cat((-right, left), -1) * sine

    return rotate(query), rotate(key)


def residency_pattern(history, block_size, recent_blocks, straddle=0.0, seed=0):
    """Which history tokens the static HBM replica holds (bool [history]).

    The most recent ``recent_blocks`` blocks are resident; then a seeded
    ``straddle`` fraction of all blocks is made half resident, so that their
    tokens come from two tiers: such a block inside the recent region loses
    its first half, one outside gains its second half. Selected blocks of
    the second kind go through the mixed-source token gather.
    """
    bs = block_size
    resident = torch.zeros(history, dtype=torch.bool)
    first = max(0, history - recent_blocks * bs)
    resident[first:] = True
    blocks = -(-history // bs)
    count = int(round(straddle * blocks))
    if count:
        g = torch.Generator().manual_seed(seed)
        for b in torch.randperm(blocks, generator=g)[:count].tolist():
            lo, mid, hi = b * bs, b * bs + bs // 2, min(history, (b + 1) * bs)
            if lo >= first:
                resident[lo:min(mid, hi)] = False
            else:
                resident[mid:hi] = True
    return resident


class NSAExtendModel:
    """Random-init NSA model whose attention runs on the B200 selected path.

    ``hot_policy``: "frequency" (the reference's hot set: the ``hot`` most
    frequently selected tokens of the last forward per layer and KV head),
    "static" (hot set left as is) or "replica" (a static HBM replica holding
    ``residency_pattern(H, BS, replica_blocks, straddle)`` of every history,
    filled during prefill, looked up through a per-token table)."""

    def __init__(self, cfg=None, *, device="cuda", seed=0, max_users=1, max_history=16384,
                 hot_policy="frequency", read_order="consumption_depth",
                 cross_query_dedup=True, pool_regions=1, chunk=1024, workspaces=None,
                 head_shard=(0, 1), exchange=None, replica_blocks=256, straddle=0.0,
                 user_workspaces=False, workspace_bytes=2 * 1024**3, attend_ctas=0):
        self.cfg = cfg = cfg or NSAConfig()
        self.device = torch.device(device)
        # KV-head sharding (the long-history serving case, one GPU pair per user): this instance owns KV heads
        # [head0, head0 + kv_local) of every layer (their query heads, pool
        # slice, cache rows, planner and attention); `exchange`
        # (sharding.PeerExchange) receives every layer's attention rows of all
        # heads: the attention launch stores this rank's rows into both GPUs'
        # gather buffers and the exchange barrier waits for the peer's.
        shard, shards = head_shard
        if shards < 1 or cfg.kv_heads % shards or not 0 <= shard < shards:
            raise ValueError("head_shard must split the KV heads evenly")
        if shards > 1 and exchange is None:
            raise ValueError("a head-sharded model needs an exchange")
        if exchange is not None and cfg.layers % 2:
            raise ValueError("the peer exchange alternates buffers by layer: even layer count")
        # user_workspaces: every user's fast path gets its own per-layer
        # transport workspaces (plan tables, staging, ready flags, counters)
        # instead of sharing one per layer, so captured graphs of different
        # users hold disjoint buffers and may run at the same time on
        # different streams (one user's host-link-bound fetch under another
        # user's projections, selection and plan). Costs one workspace per
        # (user, layer): size `workspaces` / `workspace_bytes` for that.
        self.user_workspaces = user_workspaces
        self.kv_local = cfg.kv_heads // shards
        self.head0 = shard * self.kv_local
        self.exchange = exchange
        self.max_history, self.chunk = max_history, chunk
        g = torch.Generator(device="cpu").manual_seed(seed)

        def normal(*shape):
            return (torch.randn(*shape, generator=g) * 0.02).to(torch.bfloat16).to(self.device)

        d, kvd = cfg.hidden, cfg.kv_heads * cfg.head_dim
        self.embed = normal(cfg.vocab, d)
        self.final_norm = torch.ones(d, dtype=torch.bfloat16, device=self.device)
        if cfg.compression not in ("mean", "mlp"):
            raise ValueError("compression must be 'mean' or 'mlp'")
        self.layers = []
        for _ in range(cfg.layers):
            layer = dict(
                in_norm=torch.ones(d, dtype=torch.bfloat16, device=self.device),
                post_norm=torch.ones(d, dtype=torch.bfloat16, device=self.device),
                q=normal(cfg.q_heads * cfg.head_dim, d), k=normal(kvd, d), v=normal(kvd, d),
                g=normal(cfg.q_heads * 3, d), o=normal(d, cfg.q_heads * cfg.head_dim),
                gate=normal(cfg.ffn, d), up=normal(cfg.ffn, d), down=normal(d, cfg.ffn))
            if cfg.compression == "mlp":
                # K and V compression MLPs, stacked [K, V] for batched GEMMs.
                l, hid = cfg.cmp_block, cfg.cmp_hidden
                layer.update(cmp_pe=normal(2, l, cfg.head_dim),
                             cmp_w1=normal(2, hid, l * cfg.head_dim),
                             cmp_w2=normal(2, cfg.head_dim, hid))
            self.layers.append(layer)
        self.inv_freq = 1.0 / (cfg.rope_theta ** (
            torch.arange(0, cfg.head_dim, 2, device=self.device).float() / cfg.head_dim))
        pages_per_user = cfg.layers * self.kv_local * math.ceil(max_history / 64)
        self.pool = MemoryPool(pages_per_user * max_users, 128, "host", page_size=64,
                               regions=pool_regions, device=self.device)
        self.cache = HiSparseCache(self.pool, rows=max_users * cfg.layers * self.kv_local,
                                   max_history=max_history, hot=cfg.hot,
                                   topk=min(cfg.hot, 256), dim=128)
        self.replica_blocks, self.straddle = replica_blocks, straddle
        self.resident = None  # residency pattern of the history being prefilled
        if hot_policy == "replica":
            bs = cfg.block_size
            per_row = min(max_history, replica_blocks * bs
                          + int(straddle * math.ceil(max_history / bs) + 1) * bs)
            self.cache.enable_replica(self.cache.rows * per_row)
        self.transport = GRSelectedTransport(
            self.cache, read_order=read_order, cross_query_dedup=cross_query_dedup,
            hot_policy=hot_policy, capacity=workspaces or cfg.layers + 4, async_hot=True,
            workspace_bytes=workspace_bytes, attend_ctas=attend_ctas)
        self.fast = None          # fused-glue buffers of the user being served
        self.fast_states = {}     # user -> its fused-glue buffers (prepare_fast)
        self.probe, self.probe_counters = None, []
        self.selections = None    # a list: eager fast steps append each layer's blocks
        self.layer_outputs = None  # a list: eager fast steps append each layer's output
        self.attention_outputs = None  # a list: ... and each layer's gated attention output
        self.users = {}
        self.counters = []

    # -- state -------------------------------------------------------------
    def user(self, name):
        if name not in self.users:
            cfg = self.cfg
            empty = torch.empty((0, self.kv_local, 128), dtype=torch.bfloat16, device=self.device)
            pages_needed = math.ceil(self.max_history / 64)
            self.users[name] = UserState(
                row=len(self.users) * cfg.layers * self.kv_local,
                pages=[[self.pool.allocate(pages_needed) for _ in range(self.kv_local)]
                       for _ in range(cfg.layers)],
                summaries=[empty] * cfg.layers, tails=[empty] * cfg.layers,
                windows=[empty] * cfg.layers)
        return self.users[name]

    # -- one layer -----------------------------------------------------------
    def _layer(self, index, hidden, positions, st, *, append):
        cfg, w = self.cfg, self.layers[index]
        old = st.length
        x = rms_norm(hidden, w["in_norm"], cfg.rms_eps)
        q = F.linear(x, w["q"]).view(-1, cfg.q_heads, cfg.head_dim)
        k = F.linear(x, w["k"]).view(-1, cfg.kv_heads, cfg.head_dim)
        v = F.linear(x, w["v"]).view(-1, cfg.kv_heads, cfg.head_dim)
        gates = torch.sigmoid(F.linear(x, w["g"])).view(-1, cfg.kv_heads, cfg.groups, 3)
        q, k = rotary(q, k, positions, self.inv_freq)
        own = slice(self.head0, self.head0 + self.kv_local)
        query = q.reshape(-1, cfg.kv_heads, cfg.groups, cfg.head_dim)[:, own].contiguous()
        gates = gates[:, own].contiguous()
        records = torch.cat((k[:, own], v[:, own]), -1).contiguous()
        total = old + len(records)
        if cfg.compression == "mean":
            compressed, tail = ops.append_compressed(st.summaries[index], st.tails[index],
                                                     records, cfg.block_size)
        else:
            compressed, tail = self._append_windows(w, st.summaries[index], st.tails[index],
                                                    records)
        l, d = cfg.windows
        cmp_out, blocks = ops.compressed_attention_select(
            query, compressed, positions, total, cfg.block_size, cfg.block_counts, window=l,
            stride=d, forced=cfg.forced_blocks)
        window_kv = torch.cat((st.windows[index], records))
        window_start = old - len(st.windows[index])
        base = st.row + index * self.kv_local
        fetches = [dict(row=base + h, cached_length=old, history_length=old,
                        current_kv=records[:, h].contiguous()) for h in range(self.kv_local)]
        target = None if self.exchange is None else self.exchange.targets(index, len(hidden))
        mixed, counters = self.transport.run(
            query, blocks, positions, fetches, cfg.block_size, window=cfg.window,
            window_kv=window_kv, window_start=window_start, compressed=cmp_out, gates=gates,
            output=target)
        self.counters.append(counters)
        if target is not None:
            self.exchange.barrier(torch.cuda.current_stream(self.device).cuda_stream)
        hidden = hidden + F.linear(mixed.reshape(len(hidden), -1), w["o"])
        x = rms_norm(hidden, w["post_norm"], cfg.rms_eps)
        hidden = hidden + F.linear(F.silu(F.linear(x, w["gate"])) * F.linear(x, w["up"]),
                                   w["down"])
        if append:
            self._append(index, st, records, compressed, tail, window_kv)
        return hidden

    def compress(self, w, windows):
        """MLP compression of token windows [n, l, H, 128] -> keys [n, H, 128]
        (``cxs_compress_windows``: for K and V, phi(x) = W2 silu(W1 vec(x + pe))
        with bf16 rounding after the position add, each GEMM and the silu)."""
        n, l, heads = windows.shape[:3]
        windows = windows.contiguous()
        rows = torch.arange(n * l, device=windows.device).view(n, l)
        slots = torch.arange(n, device=windows.device)
        keys = torch.empty((n, heads, windows.shape[-1]), dtype=windows.dtype,
                           device=windows.device)
        self._compress_rows(w, windows.view(n * l, heads, -1), rows, slots, keys)
        return keys

    def _compress_rows(self, w, records, rows, slots, keys, scratch=None):
        """Keys of the windows rows[i] (records row indices) into keys[slots[i]]."""
        if not len(slots):
            return
        heads, cfg = records.shape[1], self.cfg
        if scratch is None:
            scratch = torch.empty(2 * heads * len(slots) * cfg.cmp_hidden, dtype=torch.float32,
                                  device=records.device)
        _lib.check(_lib.lib().cxs_compress_windows(
            records.data_ptr(), rows.data_ptr(), len(slots), heads, cfg.cmp_block,
            cfg.cmp_hidden, w["cmp_pe"].data_ptr(), w["cmp_w1"].data_ptr(),
            w["cmp_w2"].data_ptr(), scratch.data_ptr(), keys.data_ptr(), slots.data_ptr(),
            torch.cuda.current_stream(records.device).cuda_stream))

    def _append_windows(self, w, keys, tail, records):
        """Keys of the windows that complete in tail || records (the tail
        starts at the first incomplete window) and the new tail."""
        l, d = self.cfg.windows
        values = torch.cat((tail, records))
        count = (len(values) - l) // d + 1 if len(values) >= l else 0
        if count:
            windows = values.unfold(0, l, d).permute(0, 3, 1, 2)      # [count, l, H, 128]
            keys = torch.cat((keys, self.compress(w, windows)))
        return keys, values[count * d:].clone()

    def _append(self, index, st, records, compressed, tail, window_kv):
        """Persist this chunk as history: pool write, slot table, summaries, window."""
        cfg = self.cfg
        old = st.length
        chosen = None
        if self.resident is not None:
            chosen = self.resident[old:old + len(records)].nonzero().flatten()
        for h in range(self.kv_local):
            slots = self.pool.token_slots(st.pages[index][h], old, old + len(records))
            self.pool.write_many(slots, records[:, h].contiguous(), asynchronous=True)
            self.cache.append_slots(st.row + index * self.kv_local + h, old, slots)
            if chosen is not None and len(chosen):
                self.cache.replicate(st.row + index * self.kv_local + h,
                                     (chosen + old).to(self.device),
                                     records[chosen.to(self.device), h])
        st.summaries[index], st.tails[index] = compressed, tail
        st.windows[index] = window_kv[max(0, len(window_kv) - cfg.window + 1):].clone()

    # -- public entry points -----------------------------------------------------
    def forward(self, token_ids, positions, user="user", *, append=False):
        """Run the layers over ``token_ids`` (int64, device) at ``positions``."""
        st = self.user(user)
        hidden = F.embedding(token_ids, self.embed)
        for index in range(self.cfg.layers):
            hidden = self._layer(index, hidden, positions, st, append=append)
        if append:
            st.length += len(token_ids)
        self._check_exchange()
        return rms_norm(hidden, self.final_norm, self.cfg.rms_eps)

    def _check_exchange(self):
        """Raise if a KV-head exchange barrier of this forward gave up (its
        wait is bounded; o_proj would then have read a half-filled gather
        buffer). Reads the device error word, so it synchronises; skipped
        while a CUDA graph is being captured: whoever replays the graph
        calls ``exchange.check()`` after the replay."""
        if self.exchange is not None and not torch.cuda.is_current_stream_capturing():
            self.exchange.check()

    def prefill(self, token_ids, user="user"):
        """Push a history through the model chunk by chunk, persisting its KV
        (and, with the replica policy, the resident part into the replica)."""
        st = self.user(user)
        if self.cache.replica_locs is not None:
            if st.length:
                raise ValueError("the replica policy fills a history in one prefill")
            self.resident = residency_pattern(len(token_ids), self.cfg.block_size,
                                              self.replica_blocks, self.straddle,
                                              seed=st.row)
        for begin in range(0, len(token_ids), self.chunk):
            ids = token_ids[begin:begin + self.chunk]
            positions = torch.arange(st.length, st.length + len(ids), device=self.device)
            self.forward(ids, positions, user, append=True)
            self.counters.clear()
        self.resident = None
        self.pool.flush_read_stats()
        torch.cuda.synchronize(self.device)

    def extend(self, token_ids, user="user"):
        """GR candidate suffix over the stored history (history is not appended)."""
        st = self.user(user)
        positions = torch.arange(st.length, st.length + len(token_ids), device=self.device)
        return self.forward(token_ids, positions, user, append=False)

    # -- fused-glue extend path (what the benchmark graph captures) ------------
    def prepare_fast(self, extend_tokens, user="user", candidates=1):
        """Persistent per-layer buffers for extend steps of ``extend_tokens`` tokens.

        Each layer gets a window buffer [kept + E, H, 128] whose first rows hold
        the retained history window and whose tail receives this step's K/V, a
        summaries buffer [C_hist + new, H, 128] and per-head current-KV buffers
        [H, E, 128]; the transport binds them in place (no staging copies).

        ``candidates`` > 1 serves that many GR candidates of ``extend_tokens``
        tokens each over the shared history in one step, each seeing only the
        history and its own suffix (the candidate-segment layout of
        ``cxs_attend_geometry``). The shared history ends at the last block
        boundary; the history tail past it (fewer than BS tokens) is copied
        once into the front of every candidate's segment, so each segment
        holds tail + suffix, padded to whole blocks. History blocks are then
        deduplicated across candidates, suffix blocks are candidate-private.
        """
        cfg, st, d = self.cfg, self.user(user), self.device
        E, n_cand, bs = extend_tokens, candidates, cfg.block_size
        if n_cand < 1:
            raise ValueError("candidates must be >= 1")
        rows = E * n_cand
        kl, h0, gd = self.kv_local, self.head0, cfg.groups * cfg.head_dim
        for w in self.layers:
            if "qkvg" not in w:
                # Projection rows of the owned heads only: q, k, v, gate logits.
                w["qkvg"] = torch.cat([w["q"][h0 * gd:(h0 + kl) * gd],
                                       w["k"][h0 * cfg.head_dim:(h0 + kl) * cfg.head_dim],
                                       w["v"][h0 * cfg.head_dim:(h0 + kl) * cfg.head_dim],
                                       w["g"][h0 * cfg.groups * 3:(h0 + kl) * cfg.groups * 3]]
                                      ).contiguous()
                w["gate_up"] = torch.cat([w["gate"], w["up"]]).contiguous()
                # o_proj and down as [K, N] (NN GEMMs, faster at these row
                # counts); their residual adds run in the RMSNorm that follows.
                w["o_t"] = w["o"].t().contiguous()
                w["down_t"] = w["down"].t().contiguous()
        old = st.length
        layout = SegmentLayout(old, E, n_cand, bs)
        tail_len, start, seg_tokens = layout.tail, layout.start, layout.tokens
        mlp = cfg.compression == "mlp"
        l, stride = cfg.windows
        arange_l = torch.arange(l)
        layers = []
        for index in range(cfg.layers):
            kept = len(st.windows[index])
            # mean: history records past the last complete block; mlp: past
            # the start of the first incomplete window.
            tail = len(st.tails[index])
            if tail > kept:
                raise ValueError("window must retain the summary tail")
            c_hist = len(st.summaries[index])
            base = st.row + index * kl
            last_window = (old + E - l) // stride  # last window complete by the suffix end
            if n_cand == 1:
                new = (tail + E) // bs if not mlp else max(0, last_window + 1 - c_hist)
                window_buf = torch.empty((kept + E, kl, 128), dtype=torch.bfloat16, device=d)
                window_buf[:kept] = st.windows[index]
                summaries = torch.empty((c_hist + new, kl, 128), dtype=torch.bfloat16, device=d)
                summaries[:c_hist] = st.summaries[index]
                current = torch.empty((kl, E, 128), dtype=torch.bfloat16, device=d)
                fetches = [dict(row=base + h, cached_length=old, history_length=old,
                                current_kv=current[h]) for h in range(kl)]
                entry = dict(kept=kept, tail=tail, c_hist=c_hist, new=new,
                             window_buf=window_buf, summaries=summaries, current=current,
                             fetches=fetches, window_start=old - kept)
                if mlp and new:
                    # Window i covers true positions i*d .. i*d + l - 1, at
                    # window-buffer row kept + (t - old).
                    first = torch.arange(c_hist, c_hist + new) * stride
                    entry.update(cmp_rows=(kept - old + first[:, None] + arange_l).to(d),
                                 cmp_slots=torch.arange(c_hist, c_hist + new, device=d),
                                 cmp_scratch=torch.empty(2 * kl * new * cfg.cmp_hidden,
                                                         dtype=torch.float32, device=d))
                layers.append(entry)
                continue
            if kept < tail_len:
                raise ValueError("window must retain the history tail")
            # Window buffer of a fixed length (W - 1 history records + the
            # segments), the history right-aligned against the segments: users
            # with different history lengths share workspace shapes. Records
            # before the first kept one are never inside a window.
            shared = kept - tail_len                        # window records below `start`
            lead = cfg.window - 1
            window_buf = torch.zeros((lead + n_cand * seg_tokens, kl, 128),
                                     dtype=torch.bfloat16, device=d)
            window_buf[lead - shared:lead] = st.windows[index][:shared]
            tail_records = st.windows[index][shared:]       # history past `start`
            segs = window_buf[lead:].view(n_cand, seg_tokens, kl, 128)
            segs[:, :tail_len] = tail_records
            current = torch.zeros((kl, n_cand * seg_tokens, 128), dtype=torch.bfloat16,
                                  device=d)
            current.view(kl, n_cand, seg_tokens, 128)[:, :, :tail_len] = (
                tail_records.permute(1, 0, 2)[:, None])
            fetches = [dict(row=base + h, cached_length=start, history_length=start,
                            current_kv=current[h]) for h in range(kl)]
            entry = dict(kept=lead, tail=tail_len, window_buf=window_buf, current=current,
                         fetches=fetches, window_start=start - lead)
            if not mlp:
                if c_hist * bs != start:
                    raise ValueError("layer state does not match the history length")
                nsb = seg_tokens // bs
                summaries = torch.zeros((c_hist + n_cand * nsb, kl, 128),
                                        dtype=torch.bfloat16, device=d)
                summaries[:c_hist] = st.summaries[index]
                entry.update(c_hist=c_hist, new=(tail_len + E) // bs, nsb=nsb,
                             summaries=summaries)
            else:
                # Key slots: the windows that end below `start` are shared;
                # candidate c owns seg_keys slots for its windows from seg_key
                # on (those crossing `start` and those in its segment).
                seg_key = (start - l) // stride + 1 if start >= l else 0
                seg_keys = seg_tokens // stride
                summaries = torch.zeros((seg_key + n_cand * seg_keys, kl, 128),
                                        dtype=torch.bfloat16, device=d)
                summaries[:seg_key] = st.summaries[index][:seg_key]
                static = st.summaries[index][seg_key:c_hist]  # windows inside the history
                rows_, slots_ = [], []
                for c in range(n_cand):
                    own = seg_key + c * seg_keys
                    summaries[own:own + len(static)] = static
                    for i in range(c_hist, last_window + 1):
                        t = i * stride + arange_l
                        rows_.append(torch.where(t < start, lead - (start - t),
                                                 lead + c * seg_tokens + (t - start)))
                        slots_.append(own + i - seg_key)
                entry.update(c_hist=c_hist, new=len(slots_), summaries=summaries)
                if slots_:
                    entry.update(cmp_rows=torch.stack(rows_).to(d),
                                 cmp_slots=torch.tensor(slots_, device=d),
                                 cmp_scratch=torch.empty(2 * kl * len(slots_) * cfg.cmp_hidden,
                                                         dtype=torch.float32, device=d))
            layers.append(entry)
        r = torch.arange(rows, device=d)
        true_positions = (old + r % E).to(torch.int32)
        if n_cand == 1:
            positions = true_positions
        else:
            positions = torch.tensor(layout.positions(), dtype=torch.int32, device=d)
        self.fast = self.fast_states[user] = dict(
            E=rows, per_candidate=E, candidates=n_cand, user=user, layers=layers,
            positions=positions, true_positions=true_positions, total=layout.total,
            segments=layout.segments() if n_cand > 1 else None, layout=layout,
            x=torch.empty((rows, cfg.hidden), dtype=torch.bfloat16, device=d),
            query=torch.empty((rows, kl, cfg.groups, cfg.head_dim), dtype=torch.bfloat16,
                              device=d),
            gates=torch.empty((rows, kl, cfg.groups, 3), dtype=torch.bfloat16, device=d),
            mlp=torch.empty((rows, cfg.ffn), dtype=torch.bfloat16, device=d))
        return self.fast

    def _norm(self, hidden, delta, weight, out):
        """out = rms_norm(hidden) after ``hidden += delta`` (in place, the
        residual add of the preceding projection), in one launch; plain
        rms_norm without a delta."""
        cfg, lib = self.cfg, _lib.lib()
        stream = torch.cuda.current_stream(self.device).cuda_stream
        if delta is None:
            _lib.check(lib.cxs_rms_norm(hidden.data_ptr(), weight.data_ptr(), out.data_ptr(),
                                        len(hidden), cfg.hidden, cfg.rms_eps, stream))
        else:
            _lib.check(lib.cxs_residual_rms_norm(
                hidden.data_ptr(), delta.data_ptr(), weight.data_ptr(), out.data_ptr(),
                len(hidden), cfg.hidden, cfg.rms_eps, stream))

    def _layer_fast(self, index, hidden, pending=None):
        """One layer on the fused path. ``hidden`` still lacks the previous
        layer's down projection ``pending`` (added in place by this layer's
        first RMSNorm); returns (hidden, this layer's down projection)."""
        cfg, w, f = self.cfg, self.layers[index], self.fast
        L = f["layers"][index]
        E = f["E"]
        lib = _lib.lib()
        stream = torch.cuda.current_stream(self.device).cuda_stream
        x, query, gates, positions = f["x"], f["query"], f["gates"], f["positions"]
        self._norm(hidden, pending, w["in_norm"], x)
        proj = F.linear(x, w["qkvg"])
        kl = self.kv_local
        segments = f["segments"]
        mlp = cfg.compression == "mlp"
        if segments is None:
            records = L["window_buf"][L["kept"]:]
            _lib.check(lib.cxs_qkv_rope(
                proj.data_ptr(), proj.shape[1], positions.data_ptr(), self.inv_freq.data_ptr(),
                E, kl * cfg.groups, kl, query.data_ptr(), records.data_ptr(),
                kl * 128, L["current"].data_ptr(), E * 128, gates.data_ptr(), stream))
            if L["new"] and not mlp:
                start = L["window_buf"][L["kept"] - L["tail"]:]
                _lib.check(lib.cxs_block_summaries(
                    start.data_ptr(), L["tail"] + E, kl, cfg.block_size,
                    L["summaries"][L["c_hist"]:].data_ptr(), stream))
        else:
            # Candidate c's suffix token i goes to row tail + i of segment c.
            seg_tokens, tail, per = segments[1], L["tail"], f["per_candidate"]
            records = L["window_buf"][L["kept"] + tail:]
            current = L["current"][:, tail:]
            _lib.check(lib.cxs_qkv_rope_segments(
                proj.data_ptr(), proj.shape[1], f["true_positions"].data_ptr(),
                self.inv_freq.data_ptr(), E, kl * cfg.groups, kl, query.data_ptr(),
                records.data_ptr(), kl * 128, current.data_ptr(), L["current"].shape[1] * 128,
                gates.data_ptr(), per, seg_tokens, stream))
            if L["new"] and not mlp:
                ops.block_summaries_segments(
                    L["window_buf"][L["kept"]:], tail + per, cfg.block_size,
                    L["summaries"][L["c_hist"]:], f["candidates"], seg_tokens, L["nsb"])
        if mlp and "cmp_rows" in L:
            # Keys of the windows this step completes, gathered from the window
            # buffer (history rows and the step's suffix rows) in two launches.
            self._compress_rows(w, L["window_buf"], L["cmp_rows"], L["cmp_slots"],
                                L["summaries"], L["cmp_scratch"])
        l, d = cfg.windows
        cmp_out, blocks = ops.compressed_attention_select(
            query, L["summaries"], positions, f["total"], cfg.block_size, cfg.block_counts,
            segments=segments, window=l, stride=d, forced=cfg.forced_blocks)
        if self.selections is not None:
            self.selections.append(blocks)
        if self.probe is not None:  # comparison plan on the same selections / cache state
            self.probe_counters.append(self.probe.plan_only(
                query, blocks, positions, L["fetches"], cfg.block_size, workspace_id=index))
        target = None if self.exchange is None else self.exchange.targets(index, E)
        workspace = (f["user"], index) if self.user_workspaces else index
        mixed, counters = self.transport.run(
            query, blocks, positions, L["fetches"], cfg.block_size, window=cfg.window,
            window_kv=L["window_buf"], window_start=L["window_start"], compressed=cmp_out,
            gates=gates, workspace_id=workspace, segments=segments, output=target)
        self.counters.append(counters)
        if target is not None:
            self.exchange.barrier(stream)
        if self.attention_outputs is not None:  # the transport's output is a borrowed view
            self.attention_outputs.append(mixed[:E].clone())
        # hidden = hidden + o_proj(mixed) (each rounded to bf16, as the
        # reference's bf16 tensors are), fused with the post-attention norm.
        self._norm(hidden, torch.mm(mixed.reshape(E, -1), w["o_t"]), w["post_norm"], x)
        gate_up = F.linear(x, w["gate_up"])
        _lib.check(lib.cxs_silu_mul(gate_up.data_ptr(), E, cfg.ffn, f["mlp"].data_ptr(), stream))
        return hidden, torch.mm(f["mlp"], w["down_t"])

    def extend_fast(self, token_ids, hidden=None, user=None):
        """Extend step through the fused glue (after ``prepare_fast``).

        ``hidden`` optionally replaces the token embeddings (synthetic
        candidate hidden states); ``user`` selects whose prepared buffers
        serve the step (default: the most recently prepared user)."""
        if user is not None:
            if user not in self.fast_states:
                raise ValueError(f"prepare_fast(..., user={user!r}) first")
            self.fast = self.fast_states[user]
        if self.fast is None or len(token_ids) != self.fast["E"]:
            raise ValueError("prepare_fast(len(token_ids)) first")
        # The layers update `hidden` in place; the caller's tensor stays as given.
        hidden = F.embedding(token_ids, self.embed) if hidden is None else hidden.clone()
        pending = None  # the last down projection, added by the next norm
        for index in range(self.cfg.layers):
            hidden, pending = self._layer_fast(index, hidden, pending)
            if self.layer_outputs is not None:  # materialise the layer's output
                hidden, pending = hidden + pending, None
                self.layer_outputs.append(hidden.clone())  # the next layer adds in place
        self.transport.join()
        self._check_exchange()
        out = torch.empty_like(hidden)
        self._norm(hidden, pending, self.final_norm, out)
        return out

    def capture_extend(self, extend_tokens, user="user", warmup=2, candidates=1):
        """Capture one extend forward of ``user`` in a CUDA graph with static
        input/output (``candidates`` x ``extend_tokens`` token rows, see
        ``prepare_fast``). Graphs of several users may be replayed one after
        another on one stream: they share the transport's per-layer
        workspaces, which the transport keeps (pins) once a captured graph
        holds them. With ``user_workspaces=True`` each user's graph holds its
        own workspaces (and its own graph memory pool), so graphs of
        different users may also be replayed concurrently on different
        streams; one user's graph must not overlap itself."""
        self.prepare_fast(extend_tokens, user, candidates)
        static_ids = torch.zeros(extend_tokens * candidates, dtype=torch.int64,
                                 device=self.device)
        stream = torch.cuda.Stream(self.device)
        stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(stream):
            for _ in range(warmup):
                self.counters.clear()
                self.extend_fast(static_ids)
        torch.cuda.current_stream(self.device).wait_stream(stream)
        torch.cuda.synchronize(self.device)
        self.counters.clear()
        from . import _lib

        graph = torch.cuda.CUDAGraph()
        before = _lib.lib().cxs_launch_count()
        with torch.cuda.graph(graph, stream=stream):
            static_out = self.extend_fast(static_ids)
        self.captured_launches = _lib.lib().cxs_launch_count() - before
        graph_counters = list(self.counters)
        self.counters.clear()
        # The graph reads static_ids and writes static_out in place: keep both
        # alive for as long as the graph is, whatever the caller keeps.
        graph.static_buffers = (static_ids, static_out)
        return graph, static_ids, static_out, graph_counters

    def compare_private_plan(self, token_ids, hidden=None):
        """One eager extend step that also plans each layer query-privately
        (reference QueryPrivatePlanAdapter semantics) on the same selections
        and cache state; returns (dedup misses, private misses) in tokens."""
        policy = "replica" if self.cache.replica_locs is not None else "static"
        self.probe = GRSelectedTransport(self.cache, cross_query_dedup=False,
                                         read_order="physical", hot_policy=policy,
                                         capacity=self.cfg.layers + 2)
        self.probe_counters, self.counters = [], []
        try:
            self.extend_fast(token_ids, hidden)
            torch.cuda.synchronize(self.device)
            shared = sum(int(c.statistics[:, 3].sum()) for c in self.counters)
            private = sum(int(c.statistics[:, 3].sum()) for c in self.probe_counters)
        finally:
            self.probe.close()
            self.probe, self.probe_counters = None, []
        return shared, private

    def close(self):
        self.transport.close()
        self.pool.close()
