"""Graph passes over a traced training step (:mod:`.tracer`).

Parity target: ``experiments/graph_trainer/passes.py`` (detach/identity-view cleanup,
transformer-block and automatic bucketing of FSDP collectives with reordering for overlap,
reshard-after-forward, selective activation checkpointing, CUDA graphs).  The reference hands
these jobs to Inductor's scheduler; here each pass edits the FX graph directly and the graph
is then run eagerly on the hand-written kernels, so the passes are plain node surgery:

``remove_detach``           drop ``aten.detach`` (the traced step has no autograd left)
``remove_noop_views``       drop view/reshape/expand/contiguous-clone nodes that keep the shape
``recompute_in_backward``   re-run chosen forward nodes right before their first backward use
                            instead of keeping them alive (``reshard_after_forward``: the
                            all-gathered parameters; ``selective_recompute``: everything except
                            GEMM/attention outputs and collectives)
``bucket_all_gathers``      one all-gather per bucket (flatten -> concat -> gather -> per-rank
                            column slices), issued one bucket ahead of its use (prefetch)
``bucket_reductions``       one reduce-scatter / all-reduce per bucket of gradients, waited on
                            only where the result is consumed (the optimizer inputs at the end),
                            so reductions overlap the remaining backward
``sink_waits``              move ``wait_tensor`` chains that only feed the graph output to the end

Buckets default to one per transformer block (parameter FQN ``layers.<i>.*``) plus one per
top-level module, like the reference's ``transformer_block_bucketing``;
``max_bucket_bytes`` splits larger groups (the ``auto_bucketing`` role).
"""
from __future__ import annotations

from collections import defaultdict
from typing import Callable, Iterable

import torch
import torch.fx as fx

from .tracer import TracedStep, backward_nodes

_c10d = torch.ops._c10d_functional
AG = _c10d.all_gather_into_tensor.default
RS = _c10d.reduce_scatter_tensor.default
AR = _c10d.all_reduce.default
WAIT = _c10d.wait_tensor.default
COLLECTIVES = (AG, RS, AR)
aten = torch.ops.aten


def _val(n):
    return n.meta.get("val") if isinstance(n, fx.Node) else None


def _finish(gm: fx.GraphModule) -> None:
    gm.graph.eliminate_dead_code()
    gm.graph.lint()
    gm.recompile()


def _order(gm: fx.GraphModule) -> dict[fx.Node, int]:
    return {n: i for i, n in enumerate(gm.graph.nodes)}


# --------------------------------------------------------------------------- cleanups
def remove_detach(traced: TracedStep) -> None:
    gm = traced.gm
    for n in list(gm.graph.nodes):
        if n.op == "call_function" and n.target == aten.detach.default:
            n.replace_all_uses_with(n.args[0])
            gm.graph.erase_node(n)
    _finish(gm)


_VIEWS = {aten.view.default, aten._unsafe_view.default, aten.reshape.default, aten.expand.default,
          aten.alias.default}


def remove_noop_views(traced: TracedStep) -> None:
    gm = traced.gm
    for n in list(gm.graph.nodes):
        if n.op != "call_function" or n.target not in _VIEWS or n.name == traced.loss_node:
            continue
        src, out = _val(n.args[0]), _val(n)
        if isinstance(src, torch.Tensor) and isinstance(out, torch.Tensor) and src.shape == out.shape \
                and src.stride() == out.stride():
            n.replace_all_uses_with(n.args[0])
            gm.graph.erase_node(n)
    _finish(gm)


# ------------------------------------------------------------------------ recompute
def recompute_in_backward(traced: TracedStep, should_recompute: Callable[[fx.Node], bool]) -> int:
    """For every backward use of a forward node ``a`` with ``should_recompute(a)``, re-create
    ``a`` (and, recursively, its recomputable forward inputs) right before the first backward
    user, and point all backward users at the copy.  Returns the number of copied nodes."""
    gm = traced.gm
    bwd = backward_nodes(gm, traced.loss_node)
    order = _order(gm)
    copies: dict[fx.Node, fx.Node] = {}
    first_bwd_use: dict[fx.Node, fx.Node] = {}
    for n in gm.graph.nodes:
        if n in bwd:
            for a in n.all_input_nodes:
                if a not in bwd and a.op == "call_function" and a not in first_bwd_use:
                    first_bwd_use[a] = n

    def copy(a: fx.Node, before: fx.Node) -> fx.Node:
        if a in copies:
            return copies[a]
        if a.op != "call_function" or a in bwd or not should_recompute(a):
            return a
        args = fx.node.map_arg(a.args, lambda x: copy(x, before))
        kwargs = fx.node.map_arg(a.kwargs, lambda x: copy(x, before))
        with gm.graph.inserting_before(before):
            c = gm.graph.call_function(a.target, args, kwargs)
        c.meta = dict(a.meta)
        copies[a] = c
        return c

    for a, user in sorted(first_bwd_use.items(), key=lambda kv: order[kv[1]]):
        if not should_recompute(a):
            continue
        c = copy(a, user)
        for u in list(a.users):
            if u in bwd:
                u.replace_input_with(a, c)
    _finish(gm)
    return len(copies)


def _param_derived(traced: TracedStep) -> set[fx.Node]:
    """Forward nodes computed only from parameters (casts, pads, gathers, slices, views)."""
    params = set(list(n for n in traced.gm.graph.nodes if n.op == "placeholder")[: traced.n_params])
    out = set(params)
    bwd = backward_nodes(traced.gm, traced.loss_node)
    for n in traced.gm.graph.nodes:
        if n.op == "call_function" and n not in bwd and n.all_input_nodes and \
                all(a in out for a in n.all_input_nodes):
            out.add(n)
    return out


def reshard_after_forward(traced: TracedStep) -> int:
    """Free all-gathered parameters after their forward use: backward gathers them again."""
    derived = _param_derived(traced)
    if not any(n.target == AG for n in derived):
        return 0
    return recompute_in_backward(traced, lambda n: n in derived)


_KEEP = {aten.mm.default, aten.addmm.default, aten.bmm.default, aten._scaled_dot_product_flash_attention.default,
         aten._scaled_dot_product_efficient_attention.default, aten._scaled_dot_product_cudnn_attention.default}
_KEEP_NAMES = ("tt_b200.gemm", "tt_b200.attn_fwd", "tt_b200_graph.ce_fwd")


def _expensive(n: fx.Node) -> bool:
    if n.target in _KEEP or n.target in COLLECTIVES or n.target == WAIT:
        return True
    name = str(n.target)
    return any(k in name for k in _KEEP_NAMES) or "rand" in name or "dropout" in name


def selective_recompute(traced: TracedStep) -> int:
    """Selective activation checkpointing on the graph: GEMM / attention / cross-entropy outputs
    and collectives stay alive for the backward, everything cheaper is recomputed there."""
    derived = _param_derived(traced)

    def ok(n: fx.Node) -> bool:
        if n in derived:
            return True  # parameter-derived values are recomputed by gathering (if sharded)
        return not _expensive(n) and not isinstance(_val(n), (list, tuple))

    return recompute_in_backward(traced, ok)


# ------------------------------------------------------------------------ bucketing
def default_bucket_key(fqn: str) -> str:
    parts = fqn.split(".")
    return ".".join(parts[:2]) if parts[0] == "layers" and len(parts) > 1 else parts[0]


def _source_param(n: fx.Node, ph_param: dict[str, str]) -> str | None:
    """The parameter FQN a (single-input) producer chain starts from."""
    seen = 0
    while isinstance(n, fx.Node) and seen < 64:
        if n.op == "placeholder":
            return ph_param.get(n.name)
        ins = [a for a in n.all_input_nodes]
        if len(ins) != 1:
            tensor_ins = [a for a in ins if isinstance(_val(a), torch.Tensor)]
            if len(tensor_ins) != 1:
                return None
            ins = tensor_ins
        n = ins[0]
        seen += 1
    return None


def _grad_param(wait: fx.Node, out_index: dict[fx.Node, int], names: list[str]) -> str | None:
    """The parameter whose gradient output a reduction's wait node flows into."""
    n, seen = wait, 0
    while seen < 64:
        if n in out_index:
            i = out_index[n] - 1
            return names[i] if 0 <= i < len(names) else None
        users = list(n.users)
        if len(users) != 1:
            return None
        n = users[0]
        if n.op == "output":
            return None
        seen += 1
    return None


def _hoist_producers(gm: fx.GraphModule, nodes: Iterable[fx.Node], before: fx.Node,
                     order: dict[fx.Node, int]) -> None:
    """Move the call_function ancestors of ``nodes`` that come after ``before`` to just before it
    (only chains of pure ops fed by placeholders are hoisted)."""
    todo: list[fx.Node] = []
    seen = set()

    def visit(n: fx.Node) -> None:
        if n in seen or n.op != "call_function" or order[n] < order[before]:
            return
        seen.add(n)
        for a in n.all_input_nodes:
            visit(a)
        todo.append(n)

    for n in nodes:
        visit(n)
    for n in sorted(todo, key=lambda x: order[x]):
        before.prepend(n)


def _chunks(items: list, nbytes: Callable, limit: int) -> list[list]:
    out, cur, size = [], [], 0
    for it in items:
        b = nbytes(it)
        if cur and limit > 0 and size + b > limit:
            out.append(cur)
            cur, size = [], 0
        cur.append(it)
        size += b
    if cur:
        out.append(cur)
    return out


def _numel(n: fx.Node) -> int:
    v = _val(n)
    return v.numel() if isinstance(v, torch.Tensor) else 0


def _nbytes(n: fx.Node) -> int:
    v = _val(n)
    return v.numel() * v.element_size() if isinstance(v, torch.Tensor) else 0


def bucket_all_gathers(traced: TracedStep, key_fn: Callable[[str], str] = default_bucket_key,
                       max_bucket_bytes: int = 0, prefetch: bool = True) -> int:
    """Merge the all-gathers of each bucket into one and (``prefetch``) issue every bucket's
    gather before waiting on the previous bucket's.  Returns the number of buckets built."""
    gm = traced.gm
    g = gm.graph
    bwd = backward_nodes(gm, traced.loss_node)
    ph_param = traced.placeholder_param()
    order = _order(gm)
    groups: dict[tuple, list[fx.Node]] = defaultdict(list)
    for n in g.nodes:
        if n.op != "call_function" or n.target != AG:
            continue
        waits = [u for u in n.users if u.target == WAIT]
        if len(waits) != 1 or len(n.users) != 1:
            continue
        fqn = _source_param(n.args[0], ph_param)
        if fqn is None:
            continue
        v = _val(n.args[0])
        groups[(n in bwd, key_fn(fqn), n.args[1], n.args[2], v.dtype)].append(n)
    buckets: list[list[fx.Node]] = []
    for key in sorted(groups, key=lambda k: min(order[x] for x in groups[k])):
        buckets += _chunks(groups[key], lambda n: _nbytes(n.args[0]), max_bucket_bytes)
    built = []
    for ags in buckets:
        if len(ags) == 1:
            built.append((ags[0], ags[0], next(iter(ags[0].users))))
            continue
        order = _order(gm)
        first_ag = min(ags, key=lambda x: order[x])
        _hoist_producers(gm, [a.args[0] for a in ags], first_ag, order)
        world, group = ags[0].args[1], ags[0].args[2]
        waits = [next(iter(a.users)) for a in ags]
        order = _order(gm)
        first_use = min((u for w in waits for u in w.users), key=lambda x: order[x])
        with g.inserting_before(first_ag):
            flats = [g.call_function(aten.reshape.default, (a.args[0], [-1])) for a in ags]
            cat = g.call_function(aten.cat.default, (flats, 0))
            ag = g.call_function(AG, (cat, world, group))
        with g.inserting_before(first_use):
            w = g.call_function(WAIT, (ag,))
            grid = g.call_function(aten.reshape.default, (w, [world, -1]))
            off = 0
            for a, old_w in zip(ags, waits):
                n_loc = _numel(a.args[0])
                shp = list(_val(old_w).shape)
                col = g.call_function(aten.slice.Tensor, (grid, 1, off, off + n_loc))
                full = g.call_function(aten.reshape.default, (col, shp))
                old_w.replace_all_uses_with(full)
                off += n_loc
        for old_w, a in zip(waits, ags):
            g.erase_node(old_w)
            g.erase_node(a)
        built.append((cat, ag, w))
    if prefetch:
        # issue bucket k's gather (and the ops producing its input) before waiting on bucket k-1
        _finish(gm)
        bwd = backward_nodes(gm, traced.loss_node)
        for region in (False, True):
            order = _order(gm)
            seq = sorted([b for b in built if (b[1] in bwd) == region], key=lambda b: order[b[2]])
            for prev, cur in zip(seq, seq[1:]):
                order = _order(gm)
                prev_wait = prev[2]
                if order[cur[1]] > order[prev_wait]:
                    _hoist_producers(gm, [cur[1]], prev_wait, order)
    _finish(gm)
    return len(buckets)


def _move_late_consumers(gm: fx.GraphModule, produced: list[fx.Node], out: fx.Node) -> None:
    """Consumers of ``produced`` that sit before the last produced node (an early gradient's
    post-processing, now fed by a later bucket) move right after it, in their original order."""
    order = _order(gm)
    anchor = max(produced, key=lambda n: order[n])
    late: set[fx.Node] = set()
    todo = list(produced)
    while todo:
        n = todo.pop()
        for u in n.users:
            if u is not out and u not in late and order[u] < order[anchor]:
                late.add(u)
                todo.append(u)
    for n in sorted(late, key=lambda x: order[x], reverse=True):
        anchor.append(n)


def bucket_reductions(traced: TracedStep, key_fn: Callable[[str], str] = default_bucket_key,
                      max_bucket_bytes: int = 0) -> int:
    """Merge the gradient reduce-scatters (and all-reduces) of each bucket into one collective
    issued where the bucket's last gradient is produced."""
    gm = traced.gm
    g = gm.graph
    out = next(n for n in g.nodes if n.op == "output")
    out_index = {a: i for i, a in enumerate(out.args[0]) if isinstance(a, fx.Node)}
    groups: dict[tuple, list[fx.Node]] = defaultdict(list)
    order = _order(gm)
    for n in g.nodes:
        if n.op != "call_function" or n.target not in (RS, AR):
            continue
        waits = [u for u in n.users if u.target == WAIT]
        if len(waits) != 1 or len(n.users) != 1:
            continue
        fqn = _grad_param(waits[0], out_index, traced.param_names)
        if fqn is None:
            continue
        v = _val(n.args[0])
        if n.target == RS:
            key = ("rs", key_fn(fqn), n.args[1], n.args[2], n.args[3], v.dtype)
        else:
            key = ("ar", key_fn(fqn), n.args[1], n.args[2], v.dtype)
        groups[key].append(n)
    nb = 0
    for key in sorted(groups, key=lambda k: min(order[x] for x in groups[k])):
        for colls in _chunks(groups[key], lambda n: _nbytes(n.args[0]), max_bucket_bytes):
            nb += 1
            if len(colls) == 1:
                continue
            order = _order(gm)
            last = max(colls, key=lambda x: order[x])
            waits = [next(iter(c.users)) for c in colls]
            first_use = min((u for w in waits for u in w.users), key=lambda x: order[x])
            is_rs = key[0] == "rs"
            world = colls[0].args[2] if is_rs else None
            with g.inserting_before(last.next):
                if is_rs:
                    rows = [g.call_function(aten.reshape.default, (c.args[0], [world, -1])) for c in colls]
                    cat = g.call_function(aten.cat.default, (rows, 1))
                    flat = g.call_function(aten.reshape.default, (cat, [-1]))
                    coll = g.call_function(RS, (flat,) + tuple(colls[0].args[1:]))
                else:
                    flats = [g.call_function(aten.reshape.default, (c.args[0], [-1])) for c in colls]
                    flat = g.call_function(aten.cat.default, (flats, 0))
                    coll = g.call_function(AR, (flat,) + tuple(colls[0].args[1:]))
            order = _order(gm)
            results = []
            with g.inserting_before(first_use if order[first_use] > order[coll] else out):
                w = g.call_function(WAIT, (coll,))
                off = 0
                for c, old_w in zip(colls, waits):
                    n_out = _numel(old_w)
                    piece = g.call_function(aten.slice.Tensor, (w, 0, off, off + n_out))
                    res = g.call_function(aten.reshape.default, (piece, list(_val(old_w).shape)))
                    old_w.replace_all_uses_with(res)
                    results.append(res)
                    off += n_out
            _move_late_consumers(gm, results, out)
            for old_w, c in zip(waits, colls):
                g.erase_node(old_w)
                g.erase_node(c)
    _finish(gm)
    return nb


def sink_waits(traced: TracedStep) -> int:
    """Move each ``wait_tensor`` whose transitive users only reach the graph output (gradient
    reductions) to just before the output, with that user chain."""
    gm = traced.gm
    g = gm.graph
    out = next(n for n in g.nodes if n.op == "output")
    moved = 0

    def only_to_output(n: fx.Node, chain: list[fx.Node]) -> bool:
        for u in n.users:
            if u is out:
                continue
            if u.op != "call_function" or len(u.all_input_nodes) != 1:
                return False
            chain.append(u)
            if not only_to_output(u, chain):
                return False
        return True

    for n in list(g.nodes):
        if n.op == "call_function" and n.target == WAIT:
            chain: list[fx.Node] = []
            if only_to_output(n, chain):
                for m in [n] + chain:
                    out.prepend(m)
                moved += 1
    _finish(gm)
    return moved


# ------------------------------------------------------------------------- registry
PASSES = {
    "remove_detach": lambda t, **kw: remove_detach(t),
    "remove_noop_views": lambda t, **kw: remove_noop_views(t),
    "reshard_after_forward": lambda t, **kw: reshard_after_forward(t),
    "selective_recompute": lambda t, **kw: selective_recompute(t),
    "transformer_block_bucketing": lambda t, **kw: (bucket_all_gathers(t), bucket_reductions(t), sink_waits(t)),
    "auto_bucketing": lambda t, bucket_bytes=64 << 20, **kw: (
        bucket_all_gathers(t, key_fn=lambda f: "all", max_bucket_bytes=bucket_bytes),
        bucket_reductions(t, key_fn=lambda f: "all", max_bucket_bytes=bucket_bytes), sink_waits(t)),
    "sink_waits": lambda t, **kw: sink_waits(t),
}
DEFAULT_PASSES = ["remove_detach", "remove_noop_views"]


def apply_passes(traced: TracedStep, names: list[str], **kw) -> None:
    unknown = [n for n in names if n not in PASSES]
    if unknown:
        raise ValueError(f"unknown graph passes {unknown}; available: {sorted(PASSES)}")
    for n in names:
        PASSES[n](traced, **kw)
