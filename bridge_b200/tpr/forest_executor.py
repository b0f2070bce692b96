"""Batched TPR execution of a whole forest (the training engine's hot loop).

The per-segment executor runs one segment per model forward; on a B200 that
leaves the tensor cores idle (a 512-token segment is a thin GEMM) and pays
the prefix twice (graph-free push + recomputing pop).  This engine keeps the
same relay semantics but schedules *levels of the forest*:

1. **Push, top-down** -- the internal segments of every tree at depth ``d`` run
   as packed varlen forwards of up to ``token_budget`` tokens.  Each chunk's
   post-RoPE K / raw V become per-layer *anchor* leaves (one
   ``[T_chunk, Hkv, D]`` tensor per layer, detached, ``requires_grad``).
   In ``retain`` mode (default) the chunk keeps its autograd graph and its
   owned loss; in ``recompute`` mode (the reference's memory profile) it runs
   without grad and is recomputed at pop time.
2. **Leaves** -- all leaf segments, siblings adjacent, run in packed chunks
   that attend to their parents through ``(offset, length)`` spans into the
   anchor bank (no per-sibling copies); loss + backward immediately.  The
   attention backward reduces the prefix dK/dV of all siblings into the
   anchor ``.grad`` inside the kernel.
3. **Pop, bottom-up** -- each internal chunk back-propagates
   ``[loss, K, V (, GDN states)]`` with ``[1, anchor.grad ...]``; its own prefix
   gradients land in its ancestors' anchors.

Internal segments therefore cost one forward and one backward (retain) instead
of two forwards and one backward, and every GEMM sees thousands of rows.

Parity: the event semantics of verl/models/mcore/tpr/segment_executor.py:208-444
(Push/Pop/VisitLeaf, relay of dKV and GDN dState) applied level-wise;
batching and graph retention are this framework's own design.
"""

from __future__ import annotations

from collections import defaultdict
from dataclasses import dataclass, field
from typing import Any

import numpy as np
import torch
from torch import Tensor, nn

from .context import SegmentBatchLayout, TPRAttentionContext, use_tpr_attention_context
from .prefix_state import GDNLayerState
from .segment_executor import model_device
from .tree_plan_builder import ForestExecutionPlan


@dataclass(eq=False)
class _Node:
    tree: int
    seg_id: int
    tokens: Tensor
    start: int
    depth: int
    parent: "_Node | None"
    children: list = field(default_factory=list)
    # refs owned by this node (host arrays)
    ref_rows: Tensor | None = None
    ref_targets: Tensor | None = None
    ref_samples: Tensor | None = None
    ref_flat: Tensor | None = None
    # placement after push
    chunk: "_Chunk | None" = None
    row0: int = 0
    batch_index: int = 0

    @property
    def length(self) -> int:
        return int(self.tokens.numel())

    @property
    def n_refs(self) -> int:
        return 0 if self.ref_rows is None else int(self.ref_rows.numel())


@dataclass(eq=False)
class _Chunk:
    nodes: list                                       # every node of the chunk (rank-major under CP)
    local: list = field(default_factory=list)         # the nodes this rank forwards
    counts: tuple | None = None                       # CP: (rows per rank, segments per rank)
    index: int = 0                                    # push order (deterministic on every rank)
    kv_anchor: dict = field(default_factory=dict)     # layer -> (A_K, A_V) leaves
    kv_graph: dict = field(default_factory=dict)      # layer -> (K, V) graph tensors (retain)
    gdn_anchor: dict = field(default_factory=dict)    # layer -> (A_conv, A_rec)
    gdn_graph: dict = field(default_factory=dict)
    loss: Tensor | None = None
    metrics: list = field(default_factory=list)
    offload: Any = None                               # DeferredOffload of a retained push forward


@dataclass
class ForestRunResult:
    normalized_loss: Tensor
    tree_count: int
    segment_count: int
    logical_loss_tokens: int
    forward_tokens: int
    backward_tokens: int
    chunks: int
    stats: Tensor | None
    metrics: dict


def _chunked(items: list, budget: int) -> list[list]:
    out, cur, n = [], [], 0
    for it in items:
        if cur and n + it.length > budget:
            out.append(cur)
            cur, n = [], 0
        cur.append(it)
        n += it.length
    if cur:
        out.append(cur)
    return out


class ForestExecutor:
    """Runs a :class:`ForestExecutionPlan` (PPO objective) level-wise in packed chunks."""

    def __init__(self, model: nn.Module, objective, *, mode: str = "retain", token_budget: int = 8192,
                 loss_scale: float = 1.0, cp=None, offload=None) -> None:
        """``token_budget`` is the packed token count one rank forwards at a time; ``cp`` (a
        :class:`~bridge_b200.parallel.forest_cp.ForestCP`) partitions every chunk's segments over a
        context-parallel group (chunks then hold ``token_budget * cp.size`` tokens); ``offload`` (an
        enabled :class:`~bridge_b200.tpr.activation_offload.OffloadConfig`) moves the tensors saved for
        backward to pinned host memory -- for a leaf chunk during its forward+backward, for a retained
        push chunk from its forward until its pop -- while prefix anchors and new K/V stay resident."""
        if mode not in ("retain", "recompute"):
            raise ValueError(f"mode must be 'retain' or 'recompute', got {mode!r}")
        self.model, self.objective, self.mode = model, objective, mode
        self.token_budget = int(token_budget)
        self.loss_scale = loss_scale
        self.cp = cp
        self.offload = offload if (offload is not None and offload.enabled) else None
        self._live: list[_Chunk] = []
        self.offloaded_bytes = 0
        self.before_final_backward = None   # e.g. the sharded optimizer's arm_overlap
        self._final = None                  # the chunk (or leaf group) whose backward is the step's last
        self.attn_layers = tuple(getattr(model, "attention_layer_numbers", ()))
        self.gdn_layers = tuple(getattr(model, "gdn_layer_numbers", ()))
        self.device = model_device(model)
        self.profiler = None

    # ------------------------------------------------------------------ planning
    def _nodes(self, forest: ForestExecutionPlan) -> list[_Node]:
        nodes: list[_Node] = []
        for t, tree in enumerate(forest.trees):
            plan = tree.segment_plan
            by_id: dict[int, _Node] = {}
            order = [plan.root_id]
            i = 0
            while i < len(order):
                sid = order[i]
                spec = plan.get(sid)
                parent = by_id.get(spec.parent_id) if spec.parent_id is not None else None
                node = _Node(t, sid, spec.token_ids, spec.position_start, 0 if parent is None else parent.depth + 1,
                             parent)
                if parent is not None:
                    parent.children.append(node)
                by_id[sid] = node
                nodes.append(node)
                order.extend(plan.child_ids(sid))
                i += 1
            cols = getattr(tree.objective_refs, "columns", None)
            if cols is not None:
                from .tree_plan_builder import ObjectiveRefs

                # one ref table per tree (grouped by segment), sliced per segment
                order_ = np.argsort(cols[:, 0], kind="stable")
                sorted_cols = cols[order_]
                tab = self.objective.ref_table(ObjectiveRefs(sorted_cols))
                sids, starts = np.unique(sorted_cols[:, 0], return_index=True)
                bounds = list(starts[1:]) + [len(sorted_cols)]
                for sid, a, b in zip(sids.tolist(), starts.tolist(), bounds):
                    n = by_id[sid]
                    n.ref_rows, n.ref_targets = tab.query_offsets[a:b], tab.targets[a:b]
                    n.ref_samples, n.ref_flat = tab.sample_rows[a:b], tab.flat_index[a:b]
            else:
                refs = defaultdict(list)
                for r in tree.objective_refs:
                    refs[r.segment_id].append(r)
                for sid, lst in refs.items():
                    tab = self.objective.ref_table(lst)
                    n = by_id[sid]
                    n.ref_rows, n.ref_targets, n.ref_samples, n.ref_flat = (tab.query_offsets, tab.targets,
                                                                            tab.sample_rows, tab.flat_index)
        return self._split_long(nodes)

    def _split_long(self, nodes: list[_Node]) -> list[_Node]:
        """Cut every segment longer than one rank's token budget into a chain of pieces of at most the
        budget: each piece is the parent of the next and reaches the earlier pieces as prefix K/V (and
        GDN state), exactly like a shared prefix.  No chunk then holds more than the budget, whatever the
        turn lengths, and under CP every segment can be placed whole on one rank.  Loss rows stay with
        the piece holding their query token."""
        cap = self.token_budget
        if all(n.length <= cap for n in nodes):
            return nodes
        out: list[_Node] = []
        for n in nodes:
            out.append(n)
            if n.length <= cap:
                continue
            total = n.length
            pieces = -(-total // cap)
            step = -(-total // pieces)
            tokens, children = n.tokens, n.children
            rows, tg, sm, fl = n.ref_rows, n.ref_targets, n.ref_samples, n.ref_flat
            prev = None
            for i in range(pieces):
                a, b = i * step, min(total, (i + 1) * step)
                piece = n if i == 0 else _Node(n.tree, n.seg_id, tokens[a:b], n.start + a, 0, prev)
                piece.tokens = tokens[a:b]
                piece.children = [] if i < pieces - 1 else children
                if prev is not None:
                    prev.children = [piece]
                    out.append(piece)
                if rows is not None:
                    keep = (rows >= a) & (rows < b)
                    piece.ref_rows = rows[keep] - a
                    piece.ref_targets, piece.ref_samples, piece.ref_flat = tg[keep], sm[keep], fl[keep]
                    if piece.ref_rows.numel() == 0:
                        piece.ref_rows = piece.ref_targets = piece.ref_samples = piece.ref_flat = None
                prev = piece
            for c in children:
                c.parent = prev
        # depths follow the (longer) chains
        for n in out:
            n.depth = 0
        for n in out:
            if n.parent is None:
                stack = [n]
                while stack:
                    x = stack.pop()
                    for c in x.children:
                        c.depth = x.depth + 1
                        stack.append(c)
        return out

    # ------------------------------------------------------------------ one packed forward
    def _prefix_bank(self, nodes: list[_Node]):
        """Per-layer prefix bank + spans for ``nodes`` (each attends to its full ancestor path)."""
        spans: list[tuple[int, int]] = []
        parents = [n.parent for n in nodes]
        if all(p is None for p in parents):
            return {}, [(0, 0)] * len(nodes), None
        # Fast path: every node's ancestor path is exactly one anchored chunk range (depth-1 nodes whose
        # parents are roots) and all parents live in the same pushed chunk -> the bank IS that chunk's anchors.
        chunks = {id(p.chunk): p.chunk for p in parents if p is not None}
        simple = all(p is None or p.parent is None for p in parents) and len(chunks) == 1
        if simple:
            (ch,) = chunks.values()
            for p in parents:
                spans.append((0, 0) if p is None else (p.row0, p.length))
            return {layer: ch.kv_anchor[layer] for layer in self.attn_layers}, spans, ch
        # General path: concatenate each distinct ancestor path once.
        paths: dict[int, tuple[int, int]] = {}
        pieces: list[tuple[_Chunk, int, int]] = []
        off = 0
        for p in parents:
            if p is None:
                spans.append((0, 0))
                continue
            key = id(p)
            if key not in paths:
                chain = []
                a = p
                while a is not None:
                    chain.append(a)
                    a = a.parent
                chain.reverse()
                begin = off
                for a in chain:
                    pieces.append((a.chunk, a.row0, a.length))
                    off += a.length
                paths[key] = (begin, off - begin)
            spans.append(paths[key])
        bank = {}
        for layer in self.attn_layers:
            ks = [c.kv_anchor[layer][0][r:r + n] for c, r, n in pieces]
            vs = [c.kv_anchor[layer][1][r:r + n] for c, r, n in pieces]
            bank[layer] = (torch.cat(ks), torch.cat(vs))
        return bank, spans, None

    def _gdn_init(self, nodes: list[_Node], pad_seqs: int = 0):
        if not self.gdn_layers:
            return {}
        if all(n.parent is None for n in nodes):
            return {}
        out = {}
        for layer in self.gdn_layers:
            convs, recs = [], []
            for n in nodes:
                p = n.parent
                if p is None:
                    c0, r0 = None, None
                    ref = next(x.parent for x in nodes if x.parent is not None)
                    ac, ar = ref.chunk.gdn_anchor[layer]
                    convs.append(torch.zeros_like(ac[:1]))
                    recs.append(torch.zeros_like(ar[:1]))
                else:
                    ac, ar = p.chunk.gdn_anchor[layer]
                    convs.append(ac[p.batch_index:p.batch_index + 1])
                    recs.append(ar[p.batch_index:p.batch_index + 1])
            for _ in range(pad_seqs):
                convs.append(torch.zeros_like(convs[0]))
                recs.append(torch.zeros_like(recs[0]))
            out[layer] = GDNLayerState(torch.cat(convs), torch.cat(recs))
        return out

    def _pad_multiple(self) -> int:
        if getattr(self.model, "sequence_parallel", False):
            from ..parallel.tp import tp_size

            return tp_size(self.model.tp_group)
        return 1

    def _protected(self) -> list[Tensor]:
        """Tensors offload must leave on the device: every live chunk's anchors."""
        out: list[Tensor] = []
        for ch in self._live:
            for pair in list(ch.kv_anchor.values()) + list(ch.gdn_anchor.values()):
                out.extend(pair)
        return out

    def _offload_scope(self):
        import contextlib

        if self.offload is None:
            return contextlib.nullcontext(None)
        from .activation_offload import offload_scope

        import contextlib

        @contextlib.contextmanager
        def counted():
            with offload_scope(self.model, self.offload, self._protected()) as off:
                yield off
            self.offloaded_bytes += off.offloaded_bytes

        return counted()

    def _forward(self, nodes: list[_Node], *, grad: bool, record: bool, observer=None):
        """Packed forward of ``nodes``.  A trailing pad segment (token 0, no prefix, no loss) is added
        when sequence parallelism needs the row count to divide over TP, and an idle CP rank (no
        segments in this chunk) forwards a pad segment alone so every rank makes the same collectives."""
        dev = self.device
        seq_lens = [n.length for n in nodes]
        total = sum(seq_lens)
        mult = self._pad_multiple()
        pad = (-total) % mult if nodes else max(mult, 8)
        ids_l = [n.tokens for n in nodes]
        pos_l = [torch.arange(n.start, n.start + n.length) for n in nodes]
        bank, spans, _ = self._prefix_bank(nodes)
        if pad:
            ids_l.append(torch.zeros(pad, dtype=ids_l[0].dtype if ids_l else torch.long))
            pos_l.append(torch.arange(pad))
            seq_lens.append(pad)
            spans = list(spans) + [(0, 0)]
        host = torch.stack([torch.cat(ids_l), torch.cat(pos_l)])
        if dev.type == "cuda":
            host = host.pin_memory()
        dev_ip = host.to(dev, non_blocking=True)
        layout = SegmentBatchLayout.build(seq_lens, spans, device=dev)
        gdn0 = self._gdn_init(nodes, pad_seqs=1 if pad else 0) if nodes else {}
        ctx = TPRAttentionContext(prefix_length=0, suffix_length=sum(seq_lens), past_key_values=bank,
                                  layout=layout, initial_gdn_states=gdn0,
                                  capture_gdn_final_state=record, record_new_kv=record,
                                  new_kv_observer=observer)
        max_pos = max([n.start + n.length for n in nodes] + [pad])
        with (torch.enable_grad() if grad else torch.no_grad()), use_tpr_attention_context(ctx):
            hidden = self.model(dev_ip[0], dev_ip[1], max_pos)
        return ctx, hidden

    def _exchange(self, ctx, local: list[_Node], counts):
        """This chunk's new K/V and final GDN states, restricted to real rows and (under CP) gathered
        over the CP group into rank-major anchor order."""
        rows = sum(n.length for n in local)
        segs = len(local)
        kv, gdn = {}, {}
        for layer, (k, v) in ctx.new_key_values.items():
            k, v = k[:rows], v[:rows]
            kv[layer] = (k, v) if self.cp is None else tuple(self.cp.gather([k, v], counts[0]))
        for layer, st in ctx.new_gdn_states.items():
            c, r = st.conv_state[:segs], st.recurrent_state[:segs]
            gdn[layer] = (c, r) if self.cp is None else tuple(self.cp.gather([c, r], counts[1]))
        return kv, gdn

    def _loss(self, nodes: list[_Node], hidden: Tensor):
        rows, tg, sm, fl = [], [], [], []
        base = 0
        for n in nodes:
            if n.n_refs:
                rows.append(n.ref_rows + base)
                tg.append(n.ref_targets)
                sm.append(n.ref_samples)
                fl.append(n.ref_flat)
            base += n.length
        if not rows:
            return None, None
        loss, metrics = self.objective.rows_loss(self.model, hidden, torch.cat(rows), torch.cat(tg), torch.cat(sm),
                                                 torch.cat(fl), grad_scale=self.loss_scale)
        return loss, metrics

    # ------------------------------------------------------------------ phases
    def _place(self, nodes: list[_Node]):
        """``(local nodes, rank-major order, counts)`` of a chunk (identity without CP)."""
        if self.cp is None:
            return nodes, nodes, None
        parts = self.cp.split(nodes)
        order = [n for p in parts for n in p]
        return parts[self.cp.rank], order, ([sum(n.length for n in p) for p in parts], [len(p) for p in parts])

    def _push_chunk(self, nodes: list[_Node], stats: dict, index: int = 0) -> _Chunk:
        local, order, counts = self._place(nodes)
        ch = _Chunk(order, local=local, counts=counts, index=index)
        grad = self.mode == "retain"
        row = 0
        for b, n in enumerate(order):
            n.chunk, n.row0, n.batch_index = ch, row, b
            row += n.length
        if grad and self.offload is not None:
            from .activation_offload import DeferredOffload

            ch.offload = DeferredOffload(self.model, self.offload, self._protected())
            with ch.offload.capture() as off:
                ctx, hidden = self._forward(local, grad=grad, record=True, observer=off.protect)
        else:
            ctx, hidden = self._forward(local, grad=grad, record=True)
        self._live.append(ch)
        stats["fwd"] += sum(n.length for n in local)
        kv, gdn = self._exchange(ctx, local, counts)
        for layer, (k, v) in kv.items():
            ch.kv_anchor[layer] = (k.detach().requires_grad_(True), v.detach().requires_grad_(True))
            if grad:
                ch.kv_graph[layer] = (k, v)
        for layer, (c, r) in gdn.items():
            ch.gdn_anchor[layer] = (c.detach().requires_grad_(True), r.detach().requires_grad_(True))
            if grad:
                ch.gdn_graph[layer] = (c, r)
        if grad:
            loss, metrics = self._loss(local, hidden)
            if loss is None and self.cp is not None:   # every CP rank back-propagates the whole model
                loss = hidden.float().sum() * 0.0
            ch.loss = loss
            if metrics is not None:
                ch.metrics.append(metrics)
        return ch

    def _visit_leaves(self, nodes: list[_Node], stats: dict, acc: dict) -> None:
        with self._offload_scope():
            self._visit_leaves_body(self._place(nodes)[0], stats, acc, final_key=id(nodes))

    def _visit_leaves_body(self, nodes: list[_Node], stats: dict, acc: dict, final_key=None) -> None:
        ctx, hidden = self._forward(nodes, grad=True, record=False)
        stats["fwd"] += sum(n.length for n in nodes)
        stats["bwd"] += sum(n.length for n in nodes)
        loss, metrics = self._loss(nodes, hidden)
        if loss is None:
            loss = hidden.float().sum() * 0.0
        else:
            acc["metrics"].append(metrics)
        acc["loss"] = loss.detach() if acc["loss"] is None else acc["loss"] + loss.detach()
        if self._final is final_key and self.before_final_backward is not None:
            self.before_final_backward()
        (loss * self.loss_scale).backward()

    def _pop_chunk(self, ch: _Chunk, stats: dict, acc: dict) -> None:
        import contextlib

        if ch.offload is not None:
            scope = ch.offload.backward()
        elif self.mode == "recompute":
            scope = self._offload_scope()
        else:
            scope = contextlib.nullcontext()
        with scope:
            self._pop_chunk_body(ch, stats, acc)
        if ch.offload is not None:
            self.offloaded_bytes += ch.offload.off.offloaded_bytes
        ch.offload = None
        if ch in self._live:
            self._live.remove(ch)

    def _pop_chunk_body(self, ch: _Chunk, stats: dict, acc: dict) -> None:
        if self.mode == "recompute":
            # Re-run the chunk with grad over the (still anchored) ancestors, then relay.
            ctx, hidden = self._forward(ch.local, grad=True, record=True)
            stats["fwd"] += sum(n.length for n in ch.local)
            kv_graph, gdn_graph = self._exchange(ctx, ch.local, ch.counts)
            loss, metrics = self._loss(ch.local, hidden)
            if loss is None and self.cp is not None:
                loss = hidden.float().sum() * 0.0
            if metrics is not None:
                ch.metrics.append(metrics)
        else:
            kv_graph, gdn_graph, loss = ch.kv_graph, ch.gdn_graph, ch.loss
        roots, grads = [], []
        if loss is not None:
            roots.append(loss * self.loss_scale)
            grads.append(None)
            acc["loss"] = loss.detach() if acc["loss"] is None else acc["loss"] + loss.detach()
        acc["metrics"].extend(ch.metrics)
        every = self.cp is not None      # the CP gathers' backward is a collective: every rank enters it
        for layer, (k, v) in kv_graph.items():
            ak, av = ch.kv_anchor[layer]
            if ak.grad is not None or av.grad is not None or every:
                roots += [k, v]
                grads += [ak.grad if ak.grad is not None else torch.zeros_like(ak),
                          av.grad if av.grad is not None else torch.zeros_like(av)]
        for layer, (c, r) in gdn_graph.items():
            ac, ar = ch.gdn_anchor[layer]
            if ac.grad is not None or ar.grad is not None or every:
                roots += [c, r]
                grads += [ac.grad if ac.grad is not None else torch.zeros_like(ac),
                          ar.grad if ar.grad is not None else torch.zeros_like(ar)]
        if roots:
            if self._final is ch and self.before_final_backward is not None:
                self.before_final_backward()
            torch.autograd.backward(roots, grad_tensors=grads)
        stats["bwd"] += sum(n.length for n in ch.local)
        ch.kv_anchor.clear()
        ch.kv_graph.clear()
        ch.gdn_anchor.clear()
        ch.gdn_graph.clear()
        ch.loss = None

    # ------------------------------------------------------------------ entry
    def _prof_begin(self, kind: str, nodes, depth: int):
        if self.profiler is None:
            return None
        return self.profiler.begin(kind=kind, depth=depth, tokens=sum(n.length for n in nodes))

    def _prof_end(self, rec) -> None:
        if rec is not None:
            self.profiler.end(rec)

    def plan(self, forest: ForestExecutionPlan) -> list[_Node]:
        """Static node table of a forest (reusable across runs of the same prepared batch)."""
        return self._nodes(forest)

    def run(self, forest: ForestExecutionPlan, nodes: list[_Node] | None = None) -> ForestRunResult:
        if nodes is None:
            nodes = self._nodes(forest)
        internal: dict[int, list[_Node]] = defaultdict(list)
        leaves: list[_Node] = []
        for n in nodes:
            (internal[n.depth] if n.children else leaves).append(n)
        stats = {"fwd": 0, "bwd": 0, "chunks": 0}
        acc: dict[str, Any] = {"loss": None, "metrics": []}
        pushed: dict[int, list[_Chunk]] = {}
        budget = self.token_budget * (self.cp.size if self.cp is not None else 1)
        n_pushed = 0
        for d in sorted(internal):
            pushed[d] = []
            # Keep siblings of one parent adjacent so their children batch together later.
            for grp in _chunked(internal[d], budget):
                rec = self._prof_begin("push_chunk", grp, d)
                pushed[d].append(self._push_chunk(grp, stats, n_pushed))
                self._prof_end(rec)
                n_pushed += 1
                stats["chunks"] += 1
        # Leaves ordered by (parent chunk, parent row) so a chunk's spans hit few parents.  The key is
        # the same on every rank (TP and CP peers must form identical chunks).
        leaves.sort(key=lambda n: (n.depth == 0, n.parent.chunk.index if n.parent else 0,
                                   n.parent.row0 if n.parent else 0))
        leaf_groups = _chunked(leaves, budget)
        if pushed and any(pushed.values()):
            self._final = pushed[min(pushed)][0]       # the last pop: the first chunk of the top level
        elif leaf_groups:
            self._final = id(leaf_groups[-1])
        for grp in leaf_groups:
            rec = self._prof_begin("visit_chunk", grp, grp[0].depth)
            self._visit_leaves(grp, stats, acc)
            self._prof_end(rec)
            stats["chunks"] += 1
        for d in sorted(pushed, reverse=True):
            for ch in reversed(pushed[d]):
                rec = self._prof_begin("pop_chunk", ch.nodes, d)
                self._pop_chunk(ch, stats, acc)
                self._prof_end(rec)
        loss = acc["loss"] if acc["loss"] is not None else torch.zeros((), device=self.device)
        stat_rows = [m["stats"] * m["n"] for m in acc["metrics"] if m is not None]
        total_n = sum(m["n"] for m in acc["metrics"] if m is not None)
        stats_t = (torch.stack(stat_rows).sum(0) / max(total_n, 1)) if stat_rows else None
        metrics = {"entropy_sum": sum((m["entropy_sum"] for m in acc["metrics"] if m and "entropy_sum" in m),
                                      torch.zeros((), device=self.device))} if self.objective.calculate_entropy else {}
        if self.objective.capture_log_probs:
            metrics["log_probs"] = [m.get("log_probs") for m in acc["metrics"]]
        return ForestRunResult(loss, len(forest.trees), forest.segment_count, forest.logical_loss_tokens,
                               stats["fwd"], stats["bwd"], stats["chunks"], stats_t, metrics)
