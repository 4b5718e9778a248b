"""Staging plans for a stack of Mixtral blocks (the crate's src/cluster.rs
vocabulary) and an executor that runs one on a group of processes.

`stage_mixtral(cfg, global_batch, seq, micro_batches, precision, devices)`
returns a `StagePlan` (libdop's planner, `dop_stage_mixtral`): homes,
windows in their global order, and the hops between them.  `run_plan` runs
this rank's windows in that order over torch.distributed point-to-point
messages (NCCL on GPUs, gloo on CPUs), the way the crate's `dist::run`
executes a plan (src/dist.rs:148-275) but with every device working at once:
a rank posts a window's inbound messages just before its compute and its
outbound messages right after it, grouping the sends of one window with the
receives of the next into one batch, so that two stages exchanging an
activation and an adjoint in opposite directions never wait on each other.
A message whose route passes through other devices (sparse links) is
forwarded by each of them at the consuming window: the relay receives its
hop and sends the next one at once.  Receives from a rank are posted in the
order that rank sends (`StagePlan.p2p_order`), so point-to-point matching
pairs each send with its own receive when relayed and direct messages share
a pair of ranks.
Sgd windows sum each block's adjoint over the data-parallel replicas that
hold it (an all-reduce in the replicas' group) and apply `p -= lr * dp` when
lr is not zero.  Every rank records the events it performed in the crate's
trace vocabulary (src/mixtral.rs:1393-1435); `StagePlan.rank_trace(r)` is
the plan's trace projected on rank r.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

from ._lib import check, lib

DEVICE_CPU, DEVICE_GPU = 0, 1
HOME_PARAM, HOME_TAPE = 0, 1
HOP_PARAM, HOP_ADJOINT, HOP_ACTIVATION = 0, 1, 2
PASS_FWD, PASS_BWD = 0, 1
EXEC_SGD, EXEC_BLOCK = 13, 14


class DeviceC(C.Structure):
    _fields_ = [("name", C.c_char * 32), ("kind", C.c_int32), ("pad_", C.c_int32),
                ("buffer_bytes", C.c_int64), ("code_bytes", C.c_int64)]


class LinkC(C.Structure):
    _fields_ = [("a", C.c_int32), ("b", C.c_int32)]


class HomeC(C.Structure):
    _fields_ = [(n, C.c_int32) for n in ("kind", "device", "layer", "replica", "slot", "pad_")] + [
        (n, C.c_int64) for n in ("row_begin", "row_end", "col_begin", "col_end", "stride", "bytes")]


class HopC(C.Structure):
    _fields_ = [(n, C.c_int32) for n in ("from_", "to", "kind", "pad_")] + [
        (n, C.c_int64) for n in ("bytes", "offset", "elems", "row_begin", "row_end", "col_begin",
                                 "col_end", "stride")] + [
        (n, C.c_int32) for n in ("layer", "micro", "replica", "pad2_")]


class WindowC(C.Structure):
    _fields_ = [(n, C.c_int32) for n in ("device", "pass_", "exec", "layer", "micro", "replica",
                                         "slot", "home")] + [
        (n, C.c_int64) for n in ("batch_begin", "batch_end", "resident_bytes", "tape_bytes",
                                 "param_bytes", "param_offset", "din", "dout")] + [
        ("n_inbound", C.c_int32), ("n_outbound", C.c_int32)]


@dataclass(frozen=True)
class Device:
    name: str
    kind: int = DEVICE_GPU
    buffer_bytes: int = 180 * 10**9
    code_bytes: int = 1 << 30


def b200s(n: int, buffer_bytes: int = 170 * 10**9) -> list:
    """n B200s of one box (every GPU peers every other through NVSwitch)."""
    return [Device(f"gpu{i}", DEVICE_GPU, buffer_bytes) for i in range(n)]


@dataclass(frozen=True)
class Hop:
    index: int
    src: int
    dst: int
    kind: int
    bytes: int
    rows: int
    cols: int
    layer: int
    micro: int
    replica: int


@dataclass
class Window:
    index: int
    device: int
    pass_: int
    exec: int
    layer: int
    micro: int
    replica: int
    slot: int
    batch_begin: int
    batch_end: int
    inbound: list = field(default_factory=list)
    outbound: list = field(default_factory=list)


@dataclass(frozen=True)
class Home:
    kind: int
    device: int
    layer: int
    replica: int
    slot: int
    bytes: int


def _devices_c(devices):
    arr = (DeviceC * max(1, len(devices)))()
    for i, d in enumerate(devices):
        arr[i].name = d.name.encode()[:31]
        arr[i].kind = d.kind
        arr[i].buffer_bytes = d.buffer_bytes
        arr[i].code_bytes = d.code_bytes
    return arr


def derive_links(devices) -> list:
    n = C.c_int64()
    arr = _devices_c(devices)
    check(lib().dop_derive_links(arr, len(devices), None, 0, C.byref(n)))
    out = (LinkC * max(1, n.value))()
    check(lib().dop_derive_links(arr, len(devices), out, n.value, C.byref(n)))
    return [(out[i].a, out[i].b) for i in range(n.value)]


def route_message(links, free_bytes, src: int, dst: int, nbytes: int) -> list:
    la = (LinkC * max(1, len(links)))(*[LinkC(a, b) for a, b in links])
    fa = (C.c_int64 * max(1, len(free_bytes)))(*free_bytes)
    n = C.c_int64()
    check(lib().dop_route_message(la, len(links), fa, len(free_bytes), src, dst, nbytes, None, 0,
                                  C.byref(n)))
    out = (C.c_int32 * max(1, n.value))()
    check(lib().dop_route_message(la, len(links), fa, len(free_bytes), src, dst, nbytes, out,
                                  n.value, C.byref(n)))
    return list(out[: n.value])


class StagePlan:
    def __init__(self, handle, devices):
        self._h = handle
        self.devices = list(devices)
        L = lib()
        self.hops = []
        for i in range(L.dop_plan_hop_count(self._h)):
            h = HopC()
            check(L.dop_plan_hop(self._h, i, C.byref(h)))
            self.hops.append(Hop(i, h.from_, h.to, h.kind, h.bytes, h.row_end - h.row_begin,
                                 h.col_end - h.col_begin, h.layer, h.micro, h.replica))
        self.windows = []
        for i in range(L.dop_plan_window_count(self._h)):
            w = WindowC()
            check(L.dop_plan_window(self._h, i, C.byref(w)))
            win = Window(i, w.device, w.pass_, w.exec, w.layer, w.micro, w.replica, w.slot,
                         w.batch_begin, w.batch_end)
            for outb, n, lst in ((0, w.n_inbound, win.inbound), (1, w.n_outbound, win.outbound)):
                for j in range(n):
                    k = C.c_int64()
                    check(L.dop_plan_window_hop(self._h, i, outb, j, C.byref(k)))
                    lst.append(self.hops[k.value])
            self.windows.append(win)
        self.homes = []
        for i in range(L.dop_plan_home_count(self._h)):
            h = HomeC()
            check(L.dop_plan_home(self._h, i, C.byref(h)))
            self.homes.append(Home(h.kind, h.device, h.layer, h.replica, h.slot, h.bytes))

    def __del__(self):
        try:
            if self._h:
                lib().dop_plan_destroy(self._h)
                self._h = None
        except Exception:
            pass

    def check(self, param_elems: int) -> None:
        check(lib().dop_plan_check(self._h, _devices_c(self.devices), len(self.devices),
                                   param_elems))

    def trace(self) -> list:
        n = C.c_int64()
        check(lib().dop_plan_trace(self._h, None, 0, C.byref(n)))
        buf = C.create_string_buffer(n.value + 1)
        check(lib().dop_plan_trace(self._h, buf, n.value + 1, C.byref(n)))
        return buf.value.decode().splitlines()

    def rank_trace(self, r: int) -> list:
        """The events rank r performs, in plan order: at each window its
        inbound hops (a relay on the message's route receives its hop and
        forwards the next one there), its compute, and the first hop of the
        window's outbound message when r produced it."""
        out = []
        for w in self.windows:
            for i, h in enumerate(w.inbound):
                if h.dst == r or (w.exec == EXEC_BLOCK and i > 0 and h.src == r):
                    out.append(_hop_line(h))
            if w.device == r:
                out.append(f"COMPUTE {w.device} {w.exec} {w.pass_}")
            if w.outbound and w.outbound[0].src == r:
                out.append(_hop_line(w.outbound[0]))
        return out

    def p2p_order(self) -> dict:
        """{(src, dst): hops in the order src posts them}.  A message's first
        hop is posted by its producer right after the producing window, each
        later hop by its relay at the consuming window (in route order).  A
        receiver posts its receives from src in this order, so point-to-point
        matching (which follows posting order per pair of ranks) pairs every
        send with its own receive even when relayed and direct messages share
        a pair of ranks.  Sgd inbound hops are all-reduces, not messages."""
        produced_at = {}
        for w in self.windows:
            if w.exec == EXEC_BLOCK and w.outbound:
                produced_at[w.outbound[0].index] = w.index
        posts = []
        for w in self.windows:
            if w.exec != EXEC_BLOCK or not w.inbound:
                continue
            posts.append((produced_at[w.inbound[0].index], 0, w.inbound[0]))
            posts += [(w.index, i, h) for i, h in enumerate(w.inbound) if i > 0]
        order = {}
        for _, _, h in sorted(posts, key=lambda t: (t[0], t[1])):
            order.setdefault((h.src, h.dst), []).append(h)
        return order

    def slots(self, device: int) -> dict:
        """{layer: residual slots} of the blocks homed on `device`."""
        s = {}
        for h in self.homes:
            if h.device == device and h.kind == HOME_TAPE:
                s[h.layer] = max(s.get(h.layer, 0), h.slot + 1)
        return s

    def stage_groups(self) -> list:
        """Device sets that hold the same blocks (one per pipeline stage)."""
        groups = {}
        for h in self.homes:
            if h.kind == HOME_PARAM:
                groups.setdefault(h.layer, set()).add(h.device)
        seen, out = set(), []
        for layer in sorted(groups):
            g = tuple(sorted(groups[layer]))
            if g not in seen:
                seen.add(g)
                out.append(list(g))
        return out


def _hop_line(h: Hop) -> str:
    return f"HOP {h.src} {h.dst} {h.kind} {h.bytes}"


def stage_mixtral(cfg, global_batch: int, seq: int, micro_batches: int, precision: int,
                  devices, links=None) -> StagePlan:
    h = C.c_void_p()
    la = None
    nl = 0
    if links:
        la = (LinkC * len(links))(*[LinkC(a, b) for a, b in links])
        nl = len(links)
    check(lib().dop_stage_mixtral(C.byref(cfg.to_c()), global_batch, seq, micro_batches,
                                  precision, _devices_c(devices), len(devices), la, nl,
                                  C.byref(h)))
    return StagePlan(h, devices)


def run_plan(plan: StagePlan, rank: int, lens_for, params, dparams, inputs, cotangents,
             make_buffer, lr: float = 0.0, groups=None) -> dict:
    """Run rank `rank`'s windows of `plan` (torch.distributed rank = plan
    device index).

    lens_for(layer, slot) -> lens with forward(params, x) -> y and
        backward(params, dy, dparams) -> dx (the block lens, or any lens
        with that interface)
    params[layer], dparams[layer]   this rank's blocks (dparams accumulates)
    inputs[micro]                   stack input of a micro-batch (used on the
                                    rank that runs layer 0)
    cotangents[micro]               cotangent of the stack output (used on
                                    the rank that runs the last layer)
    make_buffer(rows, cols)         an empty receive buffer
    groups                          {device tuple: process group} for the
                                    Sgd all-reduces (`stage_groups`)
    Returns {"outputs": {micro: y}, "input_grads": {micro: dx},
    "trace": [events]}.
    """
    import torch.distributed as dist

    world = dist.get_world_size() if dist.is_initialized() else 1
    if len(plan.devices) != world or not 0 <= rank < world:
        raise ValueError(f"the plan has {len(plan.devices)} devices; run_plan needs one process "
                         f"per device (world size {world}, rank {rank})")
    n_layers = 1 + max(w.layer for w in plan.windows)
    order = plan.p2p_order()
    cursor, posted = {}, set()   # per source: next hop of order[(src, rank)] to post
    arrived = {}                 # hop index -> received tensor
    acts, cots = {}, {}
    outputs, input_grads, trace = {}, {}, []
    pending = []   # (op, hop, tensor) posted at the next flush
    keep = []      # send tensors alive until their batch completes

    def flush():
        if not pending:
            return
        ops = []
        for op, h, t in pending:
            if op == "send":
                ops.append(dist.P2POp(dist.isend, t, h.dst))
            else:
                ops.append(dist.P2POp(dist.irecv, t, h.src))
        for w in dist.batch_isend_irecv(ops):
            w.wait()
        for op, h, t in pending:
            if op == "recv":
                arrived[h.index] = t
        pending.clear()
        keep.clear()

    def want(h):
        """Post the receives from h.src up to h, in the order h.src sends."""
        if h.index in posted:
            return
        seq = order[(h.src, rank)]
        k = cursor.get(h.src, 0)
        while True:
            g = seq[k]
            k += 1
            posted.add(g.index)
            pending.append(("recv", g, make_buffer(g.rows, g.cols)))
            if g.index == h.index:
                break
        cursor[h.src] = k

    for w in plan.windows:
        if w.exec == EXEC_BLOCK:
            for i, h in enumerate(w.inbound):
                if h.dst != rank:
                    continue
                want(h)
                trace.append(_hop_line(h))
                if w.device != rank:
                    # a relay on the message's route: receive, then forward
                    # the next hop at once (its receiver posts it here too)
                    flush()
                    t = arrived.pop(h.index)
                    nxt = w.inbound[i + 1]
                    pending.append(("send", nxt, t))
                    keep.append(t)
                    trace.append(_hop_line(nxt))
                    flush()
        if w.device != rank:
            continue
        if w.exec == EXEC_SGD:
            flush()
            trace += [_hop_line(h) for h in w.inbound if h.dst == rank]
            members = tuple(sorted({h.src for h in w.inbound} | {rank}))
            if len(members) > 1:
                dist.all_reduce(dparams[w.layer], group=(groups or {}).get(members))
            if lr:
                p = params[w.layer]
                p.copy_((p.float() - lr * dparams[w.layer]).to(p.dtype))
            trace.append(f"COMPUTE {w.device} {w.exec} {w.pass_}")
            continue
        flush()
        if w.inbound:
            got = arrived.pop(w.inbound[-1].index)
            (acts if w.pass_ == PASS_FWD else cots)[(w.layer, w.micro)] = got
        lens = lens_for(w.layer, w.slot)
        if w.pass_ == PASS_FWD:
            x = acts.pop((w.layer, w.micro)) if w.layer > 0 else inputs[w.micro]
            y = lens.forward(params[w.layer], x)
            if w.layer == n_layers - 1:
                outputs[w.micro] = y
            elif not w.outbound:
                acts[(w.layer + 1, w.micro)] = y
            result = y
        else:
            dy = cots.pop((w.layer, w.micro)) if w.layer < n_layers - 1 else cotangents[w.micro]
            dx = lens.backward(params[w.layer], dy, dparams[w.layer])
            if w.layer == 0:
                input_grads[w.micro] = dx
            elif not w.outbound:
                cots[(w.layer - 1, w.micro)] = dx
            result = dx
        trace.append(f"COMPUTE {w.device} {w.exec} {w.pass_}")
        if w.outbound:  # the message's first hop; relays carry the rest
            h = w.outbound[0]
            pending.append(("send", h, result))
            keep.append(result)
            trace.append(_hop_line(h))
    flush()
    return {"outputs": outputs, "input_grads": input_grads, "trace": trace}


class BlockLens:
    """A block lens for `run_plan` that runs its windows through
    `dop_run_window` (the plugin seam of the crate's `dist::Compute`,
    src/dist.rs:86-97) on one block handle (one residual slot)."""

    def __init__(self, block, stream=None):
        self.block = block
        self.stream = stream

    def _run(self, pass_, params, a, dparams=None):
        import torch
        from ._lib import ptr, stream_ptr
        w = WindowC()
        w.pass_ = pass_
        w.exec = EXEC_BLOCK
        out = torch.empty_like(a)
        check(lib().dop_run_window(self.block.handle, C.byref(w), ptr(params), ptr(a), ptr(out),
                                   ptr(dparams), stream_ptr(self.stream)))
        return out

    def forward(self, params, x):
        return self._run(PASS_FWD, params, x)

    def backward(self, params, dy, dparams):
        return self._run(PASS_BWD, params, dy, dparams)
