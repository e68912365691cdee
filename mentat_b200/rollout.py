"""Entropy-gated prefix-tree rollout on the B200 decode path.

This runs the algorithm of the reference's ``MentatGenerator.generate``
(``core/generator.py:124-245``) with this package's pieces on the hot path:

* the paged cache (``PagedKVCacheManager``: device allocator, fork, batched
  append with copy-on-write),
* tree-aware decode attention (``attn_decode``: shared prefixes read once),
* the fused gate (``Gate``: entropy, EMA, threshold, repetition penalty and the
  branch / extend decision of every active leaf in one launch and one
  device-to-host read per step, where the reference runs per-leaf Python with
  several host synchronisations, ``generator.py:333-374``).

The model stays a Hugging Face causal LM (Qwen3 or Llama family); ``PagedLM``
drives its layers the way the reference's ``PagedModelWrapper`` and adapters
do (``generator_utils.py:255-418``, ``adapters/qwen3_adapter.py``,
``adapters/llama_adapter.py``): pre-attention norm, q/k/v projections, QK-norm
on Qwen3, rotate-half RoPE at the sequence's cached length, append, attention,
o_proj, MLP, final norm and lm_head; under tensor parallelism by KV head
(``tp.py``) the attention and MLP outputs are all-reduced over the group.

``TreeRollout.generate_many`` runs several trees in lockstep, one batched
forward pass per step for the active leaves of all of them (the reference
handles one tree per ``generate``); each tree keeps its own gate state and
decisions, so every tree's result is what ``generate`` alone would give.
"""

from __future__ import annotations

import math
import time
from dataclasses import dataclass, field
from typing import Optional

import numpy as np
import torch
import torch.nn.functional as F

from . import _lib, ops
from .attention_backend import attn_decode
from .gate import Gate, GateConfig
from .paged_kv_cache import PagedKVCacheManager


# ---------------------------------------------------------------------------
# tree (generator_utils.py:40-189)
# ---------------------------------------------------------------------------
class _Hist:
    """A leaf's generated token ids as a growable int32 array (the gate's
    repetition-penalty history, handed to it without a list conversion)."""
    __slots__ = ("buf", "n")

    def __init__(self, buf=None, n: int = 0):
        self.buf = np.empty(64, np.int32) if buf is None else buf
        self.n = n

    def append(self, t: int) -> None:
        if self.n == self.buf.shape[0]:
            self.buf = np.concatenate([self.buf, np.empty_like(self.buf)])
        self.buf[self.n] = t
        self.n += 1

    def plus(self, t: int) -> "_Hist":
        h = _Hist(self.buf.copy(), self.n)
        h.append(t)
        return h

    def view(self) -> np.ndarray:
        return self.buf[: self.n]


@dataclass(eq=False)
class Node:
    node_id: int
    token_ids: list = field(default_factory=list)
    seq_id: Optional[int] = None
    parent: Optional["Node"] = None
    children: dict = field(default_factory=dict)
    cumulative_log_prob: float = 0.0
    depth: int = 0
    is_active: bool = True
    is_eos: bool = False
    sem_row: Optional[int] = None  # row of the rollout's semantic-vector table, once it has one
    entropy_ema: Optional[float] = None
    creation_step: int = 0
    is_pruned: bool = False
    # generated token ids from the root to this node (the prompt is not part),
    # kept up to date by Tree.extend / Tree.branch, as a list and as an array
    seq: list = field(default_factory=list)
    hist: _Hist = field(default_factory=_Hist)

    def full_sequence(self) -> list:
        return self.seq


class Tree:
    """Branches of one rollout, each live leaf backed by a cache sequence."""

    def __init__(self, cache: PagedKVCacheManager, sem=None):
        self.root = Node(node_id=0)
        self.cache = cache
        self.sem = sem  # the rollout's semantic-vector table (children copy their parent's row)
        self._next = 1

    def new_id(self) -> int:
        i, self._next = self._next, self._next + 1
        return i

    def extend(self, leaf: Node, token: int, log_prob: float) -> None:        # :89-99
        leaf.token_ids.append(token)
        leaf.seq.append(token)
        leaf.hist.append(token)
        leaf.cumulative_log_prob += log_prob
        leaf.depth += 1

    def branch(self, leaf: Node, tokens, log_probs) -> list:                   # :102-138
        kids = []
        for t, lp in zip(tokens, log_probs):
            child = Node(node_id=self.new_id(), token_ids=[int(t)], seq_id=self.cache.fork_sequence(leaf.seq_id),
                         parent=leaf, cumulative_log_prob=leaf.cumulative_log_prob + float(lp), depth=leaf.depth + 1,
                         entropy_ema=leaf.entropy_ema, seq=leaf.seq + [int(t)], hist=leaf.hist.plus(int(t)))
            if leaf.sem_row is not None and self.sem is not None:
                child.sem_row = self.sem.copy_row(leaf.sem_row)
            leaf.children[child.node_id] = child
            kids.append(child)
        leaf.is_active = False
        if leaf.seq_id is not None:
            self.cache.free_sequence(leaf.seq_id)
            leaf.seq_id = None
        return kids

    def prune(self, node: Node) -> None:                                       # :141-169
        if node.seq_id is not None:
            self.cache.free_sequence(node.seq_id)
            node.seq_id = None
        node.is_active = False
        node.is_pruned = True
        p = node.parent
        if p is not None and not p.is_active and p.parent is not None and \
                all(c.is_pruned for c in p.children.values()):
            self.prune(p)

    def active_leaves(self) -> list:                                           # :171-189
        out = []
        self._walk(self.root, out, True)
        return out

    def finished(self) -> list:
        out = []
        self._walk(self.root, out, False)
        return out

    def _walk(self, node: Node, out: list, active: bool) -> None:
        if active:
            if node.is_active and not node.children and not node.is_eos:
                out.append(node)
        elif node.is_eos:
            out.append(node)
        for c in node.children.values():
            self._walk(c, out, active)

    def free_all(self) -> None:
        stack = [self.root]
        while stack:
            n = stack.pop()
            if n.seq_id is not None:
                self.cache.free_sequence(n.seq_id)
                n.seq_id = None
            stack.extend(n.children.values())


# ---------------------------------------------------------------------------
# model driver (generator_utils.py:255-418, adapters/*_adapter.py)
# ---------------------------------------------------------------------------
class PagedLM:
    """Runs a Hugging Face Qwen3 / Llama causal LM over the paged cache."""

    def __init__(self, model, cache: PagedKVCacheManager, tp_group=None):
        base = model.model
        self.model, self.cache = model, cache
        # tensor parallelism by KV head (``tp.shard_model``): the attention and MLP
        # outputs are partial sums over the group, all-reduced before the residual
        self.tp_group = tp_group
        self.embed, self.layers, self.norm, self.lm_head = base.embed_tokens, base.layers, base.norm, model.lm_head
        self.rotary = base.rotary_emb
        cfg = model.config
        self.hq, self.hkv = cfg.num_attention_heads, cfg.num_key_value_heads
        self.hd = getattr(cfg, "head_dim", None) or cfg.hidden_size // self.hq
        self.qk_norm = hasattr(self.layers[0].self_attn, "q_norm")  # Qwen3

    def _sum(self, x: torch.Tensor) -> torch.Tensor:
        if self.tp_group is not None:
            torch.distributed.all_reduce(x, group=self.tp_group)
        return x

    @staticmethod
    def _rope(t, cos, sin):
        h = t.shape[-1] // 2
        return t * cos + torch.cat((-t[..., h:], t[..., :h]), dim=-1) * sin

    def _qkv(self, attn, x, shape):
        q = attn.q_proj(x).view(*shape, self.hq, self.hd)
        k = attn.k_proj(x).view(*shape, self.hkv, self.hd)
        v = attn.v_proj(x).view(*shape, self.hkv, self.hd)
        if self.qk_norm:
            q, k = attn.q_norm(q), attn.k_norm(k)
        return q, k, v

    @torch.no_grad()
    def prefill(self, input_ids: torch.Tensor, seq_id: int) -> torch.Tensor:
        """The prompt (L,) into the cache of ``seq_id``; logits (V,) of its last position."""
        L = input_ids.shape[-1]
        h = self.embed(input_ids.view(1, L))
        pos = torch.arange(L, device=h.device).view(1, L)
        cos, sin = self.rotary(h, pos)
        cos, sin = cos.unsqueeze(2), sin.unsqueeze(2)  # (1, L, 1, hd)
        for layer_idx, blk in enumerate(self.layers):
            attn = blk.self_attn
            q, k, v = self._qkv(attn, blk.input_layernorm(h), (1, L))
            q, k = self._rope(q, cos, sin), self._rope(k, cos, sin)
            self.cache.append_tokens(seq_id, layer_idx, k[0], v[0])
            o = self.cache.prefill_attention(seq_id, layer_idx, q[0]).view(1, L, self.hq, self.hd)
            h = h + self._sum(attn.o_proj(o.reshape(1, L, -1)))
            h = h + self._sum(blk.mlp(blk.post_attention_layernorm(h)))
        return self.lm_head(self.norm(h)[0, -1])

    # ---- CUDA-graph decode ----------------------------------------------------
    # One graph per number of sequences N captures the whole multi-layer decode
    # step: embedding, every layer (the append and decode operators included)
    # and the lm_head.  The token ids and cache slots are static buffers filled
    # before a replay; RoPE positions are read on the device from the cache's
    # lengths, and the decode kernels plan from the device tables, so a replay
    # needs no host work beyond the host mirror of the lengths.
    _graphs = None

    def enable_graphs(self, max_len: int, max_n: int, bucket: Optional[int] = None) -> None:
        """Decode through CUDA graphs; ``max_len`` bounds every sequence's length
        and ``max_n`` the sequences of one step (they size the shared workspace,
        which captured graphs must not see reallocated).  With ``bucket``, a step
        of N sequences replays the graph of N rounded up to a multiple of
        ``bucket``: the extra rows append nothing (slot -1) and attend over an
        empty sequence, so a few graphs cover every leaf count."""
        self._bucket = bucket
        if bucket:
            max_n = -(-max_n // bucket) * bucket
            if self._pad_seq is None:
                self._pad_seq = self.cache.allocate_sequence()  # never appended to: length 0
        self.cache.decode_workspace(max_n, self.hq, max_len)
        self.cache.pin_workspace()
        self._graph_max_len = max_len
        self._graph_max_n = max_n
        self._graphs = {}
        self._pool = torch.cuda.graph_pool_handle()

    _bucket = None
    _pad_seq = None

    def _forward_static(self, tokens: torch.Tensor, slots: torch.Tensor,
                        dec_slots: Optional[torch.Tensor] = None) -> tuple:
        """One decode step over static buffers; ``slots`` receive the new K/V rows,
        ``dec_slots`` (default ``slots``) are the sequences attended over."""
        c = self.cache
        N = tokens.shape[0]
        if dec_slots is None:
            dec_slots = slots
        h = self.embed(tokens)
        pos = c._ntok[0].index_select(0, dec_slots).to(torch.long).view(N, 1)  # lengths before this token
        cos, sin = self.rotary(h, pos)
        scale = 1.0 / (self.hd ** 0.5)
        for layer_idx, blk in enumerate(self.layers):
            attn = blk.self_attn
            q, k, v = self._qkv(attn, blk.input_layernorm(h), (N,))
            q, k = self._rope(q, cos, sin), self._rope(k, cos, sin)
            ops.append_batched(c._k_all, c._v_all, slots, k, v, c._op_id, layer_idx)
            # every layer has the tree's sharing structure: plan once per step
            o = ops.paged_decode(q, dec_slots, self._graph_max_len, c._op_id, layer_idx, scale,
                                 reuse_plan=layer_idx > 0)
            h = h + self._sum(attn.o_proj(o.reshape(N, -1)))
            h = h + self._sum(blk.mlp(blk.post_attention_layernorm(h)))
        h = self.norm(h)
        return self.lm_head(h), h

    # kernels of this library run by graph replays (a replay launches no kernel
    # from the host, so the library's own launch counter does not see them)
    graph_kernel_launches = 0

    def _capture(self, N: int) -> dict:
        dev = self.cache.device
        g = {"tokens": torch.zeros(N, dtype=torch.long, device=dev),
             "slots": torch.full((N,), -1, dtype=torch.int32, device=dev),
             "dec_slots": torch.zeros(N, dtype=torch.int32, device=dev) if self._bucket else None,
             "graph": torch.cuda.CUDAGraph()}
        if self._bucket:
            g["dec_slots"].fill_(self.cache._sequences[self._pad_seq].slot)
        lib = _lib.load()
        n0 = lib.mentat_kernel_launch_count()
        with torch.cuda.graph(g["graph"], pool=self._pool):
            g["logits"], g["hidden"] = self._forward_static(g["tokens"], g["slots"], g["dec_slots"])
        g["kernels"] = lib.mentat_kernel_launch_count() - n0
        self._graphs[N] = g
        return g

    # Static eager decode: the graph path's forward run without capture, for
    # batches whose many distinct sizes would each need a graph.  It plans
    # from the device tables like a replay, so a step has no per-layer host work.
    _static_max_len = None

    def enable_static(self, max_len: int) -> None:
        self._graph_max_len = max_len
        self._static_max_len = max_len

    @torch.no_grad()
    def decode(self, tokens: torch.Tensor, seq_ids: list) -> tuple:
        """One token per sequence: logits (N, V) and final hidden states (N, D)."""
        N = len(seq_ids)
        seq = self.cache._sequences
        # captured and static steps size their workspace for _graph_max_len tokens
        # (the new one included); longer sequences take the eager path
        fits = (self._graphs is not None or self._static_max_len is not None) and \
            max(seq[s].num_tokens[0] for s in seq_ids) < self._graph_max_len
        if fits and self._graphs is not None and N <= self._graph_max_n:
            if self._bucket:
                Nb = -(-N // self._bucket) * self._bucket
                g = self._graphs.get(Nb) or self._capture(Nb)
                # the padding rows: token 0, no append (slot -1), attention over the empty sequence
                pad = seq[self._pad_seq].slot
                sl = [seq[s].slot for s in seq_ids]
                both = torch.tensor([sl + [-1] * (Nb - N), sl + [pad] * (Nb - N)], dtype=torch.int32)
                up = self.cache._uploads.upload(both.view(-1)).view(2, Nb)
                g["tokens"][:N].copy_(tokens.view(N))
                g["tokens"][N:].zero_()
                g["slots"].copy_(up[0])
                g["dec_slots"].copy_(up[1])
            else:
                g = self._graphs.get(N) or self._capture(N)
                g["tokens"].copy_(tokens.view(N))
                g["slots"].copy_(self.cache._slots_dev(seq_ids))
            g["graph"].replay()
            self.graph_kernel_launches += g["kernels"]
            self.cache.mirror_decode_step(seq_ids)
            return g["logits"][:N], g["hidden"][:N]
        if fits and self._static_max_len is not None:
            out = self._forward_static(tokens.view(N), self.cache._slots_dev(seq_ids))
            self.cache.mirror_decode_step(seq_ids)
            return out
        h = self.embed(tokens.view(N))
        pos = torch.tensor([self.cache.get_kv_length(s) for s in seq_ids], device=h.device).view(N, 1)
        cos, sin = self.rotary(h, pos)  # (N, 1, hd): broadcasts over heads
        for layer_idx, blk in enumerate(self.layers):
            attn = blk.self_attn
            q, k, v = self._qkv(attn, blk.input_layernorm(h), (N,))
            q, k = self._rope(q, cos, sin), self._rope(k, cos, sin)
            # the new token's K/V go in first, so it attends to itself
            self.cache.append_tokens_batched(seq_ids, layer_idx, k, v)
            pk, pv, cu, mx = self.cache.build_packed_kv(seq_ids, layer_idx)
            o = attn_decode(q, pk, pv, None, cu, mx, N)
            h = h + self._sum(attn.o_proj(o.reshape(N, -1)))
            h = h + self._sum(blk.mlp(blk.post_attention_layernorm(h)))
        h = self.norm(h)
        return self.lm_head(h), h


# ---------------------------------------------------------------------------
# semantic vectors (generator.py:376-398, 400-497)
# ---------------------------------------------------------------------------
class _SemTable:
    """Every node's semantic vector, one row each of a device table: the EMA of
    the leaf's final hidden states over its decode steps.  A branch's children
    start from copies of the parent's row; the copies of a step are batched and
    run before the next read of the table."""

    def __init__(self, dim: int, dtype, device, cap: int = 256):
        self.t = torch.empty((cap, dim), dtype=dtype, device=device)
        self.n = 0
        self._copies = []

    def _alloc(self) -> int:
        if self.n == self.t.shape[0]:
            t = torch.empty((2 * self.n, self.t.shape[1]), dtype=self.t.dtype, device=self.t.device)
            t[: self.n].copy_(self.t)
            self.t = t
        r, self.n = self.n, self.n + 1
        return r

    def _idx(self, rows) -> torch.Tensor:
        return torch.tensor(rows, dtype=torch.long).to(self.t.device, non_blocking=True)

    def copy_row(self, src: int) -> int:
        dst = self._alloc()
        self._copies.append((src, dst))
        return dst

    def flush(self) -> None:
        if self._copies:
            src, dst = zip(*self._copies)
            self.t.index_copy_(0, self._idx(dst), self.t.index_select(0, self._idx(src)))
            self._copies = []

    def update(self, leaves, hidden: torch.Tensor, alpha: float) -> None:
        """First step of a leaf: its hidden state; later: (1 - a) v + a h, with the
        reference's two rounded steps (``v.mul_(1 - a).add_(h, alpha=a)``)."""
        self.flush()
        new_i, new_r, upd_i, upd_r = [], [], [], []
        for i, lf in enumerate(leaves):
            if lf.sem_row is None:
                lf.sem_row = self._alloc()
                new_i.append(i)
                new_r.append(lf.sem_row)
            else:
                upd_i.append(i)
                upd_r.append(lf.sem_row)
        if new_i:
            self.t.index_copy_(0, self._idx(new_r), hidden.index_select(0, self._idx(new_i)))
        if upd_i:
            rows = self._idx(upd_r)
            v = self.t.index_select(0, rows)
            v.mul_(1.0 - alpha).add_(hidden.index_select(0, self._idx(upd_i)), alpha=alpha)
            self.t.index_copy_(0, rows, v)

    def rows(self, rows) -> torch.Tensor:
        self.flush()
        return self.t.index_select(0, self._idx(rows))


# ---------------------------------------------------------------------------
# rollout (generator.py:54-497)
# ---------------------------------------------------------------------------
class TreeRollout:
    """The entropy-gated tree rollout of ``MentatGenerator`` (same knobs and defaults)."""

    def __init__(self, model, *, eos_token_id=2, max_active_branches: int = 10, branching_factor: int = 3,
                 relative_entropy_multiplier: float = 1.25, entropy_ema_alpha: float = 0.3,
                 max_new_tokens: int = 256, temperature: float = 0.7, repetition_penalty: float = 1.2,
                 block_size: int = 16, max_blocks: int = 8192, semantic_similarity_threshold: float = 0.85,
                 ema_alpha: float = 0.3, min_steps_before_prune: int = 5, soft_explore_window: int = 10,
                 soft_explore_initial: float = 0.3, max_seqs: int = 256, cuda_graphs: bool = True,
                 max_prompt_len: int = 4096, entropy_threshold: Optional[float] = None,
                 max_blocks_per_seq: Optional[int] = None, static_decode: bool = False, tp_group=None,
                 graph_bucket: Optional[int] = None, log_softmax: str = "cpu"):
        cfg = model.config
        dev = next(model.parameters()).device
        dtype = next(model.parameters()).dtype
        hq = cfg.num_attention_heads
        hd = getattr(cfg, "head_dim", None) or cfg.hidden_size // hq
        self.cache = PagedKVCacheManager(cfg.num_hidden_layers, cfg.num_key_value_heads, hd, max_blocks, block_size,
                                         dev, dtype, max_seqs=max_seqs, max_blocks_per_seq=max_blocks_per_seq)
        self.lm = PagedLM(model, self.cache, tp_group)
        self.eos = set(eos_token_id) if isinstance(eos_token_id, (list, tuple)) else {eos_token_id}
        self.M, self.K = max_active_branches, branching_factor
        self.max_new_tokens = max_new_tokens
        self.sim_threshold, self.ema_alpha = semantic_similarity_threshold, ema_alpha
        self.min_steps_before_prune = min_steps_before_prune
        self.gate_cfg = GateConfig(temperature=temperature, repetition_penalty=repetition_penalty,
                                   entropy_ema_alpha=entropy_ema_alpha,
                                   relative_entropy_multiplier=relative_entropy_multiplier,
                                   soft_explore_initial=soft_explore_initial, branching_factor=branching_factor,
                                   max_active_branches=max_active_branches, soft_explore_window=soft_explore_window,
                                   pen_entropy=False,  # only the reference's diagnostics use it
                                   log_softmax=log_softmax)
        self.device = dev
        self.cuda_graphs = cuda_graphs
        self.static_decode = static_decode  # without graphs: plan on the device, no per-layer host work
        self.graph_bucket = graph_bucket    # graphs for leaf counts rounded up to a multiple of this
        self.max_prompt_len = max_prompt_len
        # A fixed entropy threshold replaces the adaptive one in the branch test
        # (the benchmark configurations calibrate it on a warm-up rollout); the
        # room test M - n >= K stays.  entropy_log, when a list, collects every
        # leaf's float-accurate gate entropy.
        self.entropy_threshold = entropy_threshold
        self.entropy_log = None
        self.decode_tokens = 0       # one per active leaf per decode step (step 0 excluded)
        self.decode_time_s = 0.0
        self.steps = 0
        self.step_leaves = []        # sequences decoded at each step
        self.trace = None            # when a list: each step's active leaves (generated ids), per tree

    # ---- per-leaf decision (generator.py:250-374) ---------------------------
    def _records(self, recs) -> list:
        """The gate records of a step as plain tuples (ema, accurate entropy, branch,
        argmax, argmax log-prob, top-K ids, top-K log-probs), one column at a time."""
        K = self.K
        return list(zip(recs["ema"].tolist(), recs["entropy_acc"].tolist(), recs["branch"].tolist(),
                        recs["argmax"].tolist(), recs["argmax_lp"].tolist(), recs["topk_ids"][:, :K].tolist(),
                        recs["topk_lps"][:, :K].tolist()))

    def _apply(self, tree: Tree, leaf: Node, rec, step: int, n_active: int) -> None:
        ema, h_acc, branch, arg, arg_lp, top_ids, top_lps = rec
        leaf.entropy_ema = ema
        if self.entropy_log is not None:
            self.entropy_log.append(h_acc)
        if self.entropy_threshold is not None:
            # the fixed threshold is compared with the float-accurate entropy: the
            # bf16-rounded one takes few distinct values (0.0625 apart near 11 nats)
            branch = h_acc > self.entropy_threshold and self.M - n_active >= self.K
        if branch:
            kids = tree.branch(leaf, top_ids, top_lps)
            for c in kids:
                c.creation_step = step
                self._eos(c)
        else:
            tree.extend(leaf, arg, arg_lp)
            self._eos(leaf)

    def _eos(self, node: Node) -> None:
        if node.token_ids[-1] in self.eos:
            node.is_eos, node.is_active = True, False
            if node.seq_id is not None:
                self.cache.free_sequence(node.seq_id)
                node.seq_id = None

    def _prune_similar(self, trees, step: int) -> None:                       # :400-497
        """Semantic pruning of every tree of the step: one normalize + mm over the
        warmed-up leaves of all trees, then ``mentat_prune_similar`` masks each
        tree's pairs (upper triangle, no siblings, none across trees) and resolves
        them in the reference's row-major order on the device; the host reads one
        flag per leaf and prunes in the reference's leaf order."""
        groups = []
        for tree in trees:
            cand = [lf for lf in tree.active_leaves()
                    if lf.sem_row is not None and step - lf.creation_step >= self.min_steps_before_prune]
            if len(cand) > 1:
                groups.append((tree, cand))
        if not groups:
            return
        flat = [lf for _, cand in groups for lf in cand]
        v = F.normalize(self.sem.rows([lf.sem_row for lf in flat]), p=2, dim=1)
        sim = v @ v.t()
        off = np.zeros(len(groups) + 1, np.int64)
        np.cumsum([len(cand) for _, cand in groups], out=off[1:])
        # one host buffer: group offsets, parent keys, cumulative log-probs (8 bytes each)
        host = np.empty(len(off) + 2 * len(flat), np.int64)
        host[: len(off)] = off
        host[len(off): len(off) + len(flat)] = [id(lf.parent) if lf.parent is not None else -1 - i
                                                for i, lf in enumerate(flat)]
        host[len(off) + len(flat):].view(np.float64)[:] = [lf.cumulative_log_prob for lf in flat]
        dev = torch.from_numpy(host).to(sim.device, non_blocking=True)
        flags = ops.prune_similar(sim, dev[: len(off)].to(torch.int32), dev[len(off): len(off) + len(flat)],
                                  dev[len(off) + len(flat):].view(torch.float64), self.sim_threshold,
                                  max(len(cand) for _, cand in groups)).cpu().numpy()
        for g, (tree, cand) in enumerate(groups):
            for k, lf in enumerate(cand):
                if flags[off[g] + k] and lf.is_active:
                    tree.prune(lf)

    # ---- rollout -------------------------------------------------------------
    def generate(self, prompt_ids) -> list:
        return self.generate_many([prompt_ids])[0]

    def generate_many(self, prompts) -> list:
        """Rolls out one tree per prompt (token-id sequences), all in lockstep."""
        trees, gates = [], []
        self.sem = _SemTable(self.lm.model.config.hidden_size, next(self.lm.model.parameters()).dtype, self.device)
        for p in prompts:
            ids = torch.as_tensor(p, dtype=torch.long, device=self.device)
            sid = self.cache.allocate_sequence()
            logits = self.lm.prefill(ids, sid)
            tree = Tree(self.cache, self.sem)
            first = Node(node_id=tree.new_id(), seq_id=sid, parent=tree.root)
            tree.root.children[0] = first
            gate = Gate(self.device, self.gate_cfg)
            gate.launch(logits.view(1, -1), [[]], [None], num_active=1, step=0)
            self._apply(tree, first, self._records(gate.result())[0], 0, 1)
            trees.append(tree)
            gates.append(gate)
        longest = max(max(len(p) for p in prompts), self.max_prompt_len) + self.max_new_tokens + 1
        if self.cuda_graphs and self.lm._graphs is None:
            # a step decodes at most every tree's live leaves, which stay within
            # max_active_branches + the K - 1 extra children of a last branch each
            self.lm.enable_graphs(longest, min(self.cache.max_seqs - 1, len(prompts) * (self.M + self.K * self.M)),
                                  self.graph_bucket)
        elif self.static_decode and self.lm._graphs is None and self.lm._static_max_len is None:
            self.lm.enable_static(longest)
        torch.cuda.synchronize(self.device)
        t0 = time.perf_counter()
        for step in range(1, self.max_new_tokens):
            per_tree = [t.active_leaves() for t in trees]
            leaves = [lf for lv in per_tree for lf in lv]
            if not leaves:
                break
            self.steps += 1
            self.step_leaves.append(len(leaves))
            if self.trace is not None:
                self.trace.append([sorted(list(lf.seq) for lf in lv) for lv in per_tree])  # copies: leaves grow
            tokens = torch.tensor([lf.token_ids[-1] for lf in leaves], dtype=torch.long).to(self.device,
                                                                                              non_blocking=True)
            logits, hidden = self.lm.decode(tokens, [lf.seq_id for lf in leaves])
            self.decode_tokens += len(leaves)
            self.sem.update(leaves, hidden, self.ema_alpha)                    # :376-398
            if self.entropy_threshold is None:
                # adaptive threshold: one gate launch per tree (the threshold uses the
                # tree's active count), then one wait
                a = 0
                for lv, gate in zip(per_tree, gates):
                    if lv:
                        gate.launch(logits[a:a + len(lv)], [lf.hist.view() for lf in lv],
                                    [lf.entropy_ema for lf in lv], num_active=len(lv), step=step)
                    a += len(lv)
                recs_of = [self._records(gate.result()) if lv else None for lv, gate in zip(per_tree, gates)]
            else:
                # fixed threshold: the host takes the decision from the entropy, so one
                # launch covers the leaves of every tree
                gates[0].launch(logits[:len(leaves)], [lf.hist.view() for lf in leaves],
                                [lf.entropy_ema for lf in leaves], num_active=len(leaves), step=step)
                recs_all = self._records(gates[0].result())
                recs_of, a = [], 0
                for lv in per_tree:
                    recs_of.append(recs_all[a:a + len(lv)])
                    a += len(lv)
            for tree, lv, recs in zip(trees, per_tree, recs_of):
                for lf, rec in zip(lv, recs if lv else ()):
                    if lf.is_active:
                        self._apply(tree, lf, rec, step, len(lv))
            self._prune_similar(trees, step)
        torch.cuda.synchronize(self.device)
        self.decode_time_s += time.perf_counter() - t0
        out = []
        for tree in trees:
            res = []
            for node in tree.finished() + tree.active_leaves():
                tids = node.full_sequence()
                res.append({"token_ids": tids, "log_prob": node.cumulative_log_prob,
                            "norm_prob": math.exp(node.cumulative_log_prob / max(len(tids), 1))})
            tree.free_all()
            res.sort(key=lambda r: r["norm_prob"], reverse=True)
            out.append(res)
        return out

    def calibrate_threshold(self, prompts, steps: int = 32, q: float = 90.0) -> float:
        """Sets the fixed entropy threshold to the q-th percentile of the gate
        entropies of a ``steps``-step rollout of ``prompts`` without branching;
        returns it.  The counters of that rollout are discarded."""
        keep = (self.max_new_tokens, self.decode_tokens, self.decode_time_s, self.steps, self.cuda_graphs,
                self.static_decode, list(self.step_leaves))
        self.entropy_threshold, self.entropy_log = math.inf, []
        # host-planned steps: graphs or the static path set up now would size their
        # workspace for this short rollout
        self.max_new_tokens, self.cuda_graphs, self.static_decode = steps + 1, False, False
        try:
            self.generate_many(prompts)
            log = self.entropy_log[len(prompts):]  # the decode steps (step 0 is the prompt's own)
        finally:
            (self.max_new_tokens, self.decode_tokens, self.decode_time_s, self.steps, self.cuda_graphs,
             self.static_decode, self.step_leaves) = keep
            self.entropy_log = None
        self.entropy_threshold = float(np.percentile(np.asarray(log, np.float64), q))
        return self.entropy_threshold

    def tree_tokens_per_s(self) -> float:
        """Decode tokens per second of decode wall time (``generator.py:508-511``)."""
        return self.decode_tokens / self.decode_time_s if self.decode_time_s > 0 else 0.0
