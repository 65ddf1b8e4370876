"""Executable model of the synchronisation protocol of the tensor-core stencil forward.

The kernel (``pack3d_b200/csrc/stencil_fwd.cu``) coordinates one TMA producer thread,
one MMA-issuing thread and eight softmax warps through mbarriers that are waited on by
*phase parity*.  A parity wait cannot count: it passes when the barrier's current phase
parity differs from the awaited one, and a freshly initialised barrier reports its
"preceding phase" (parity 1) as complete.  This module replays that protocol step by
step -- every role as a program, TMA copies and tensor-core operations as asynchronous
events that complete later (MMAs in issue order) -- under random interleavings, with
the hardware's parity semantics, and checks:

* every wait passes only once the completion it stands for has happened;
* no barrier gets an arrival while its pending count is zero (an over-arrival);
* a ring stage is overwritten only after every MMA that reads its previous chunk has
  completed, and is read only after its copy has landed;
* a TMEM S buffer is rewritten only after the PV MMA reading its P has completed, P is
  read by PV only after the four softmax warps stored it, and O is read or rescaled only
  between PV completions;
* every role finishes (no deadlock).

The model mirrors the kernel's barrier map and wait parities one for one; a change to
either must be made in both.  ``release="sready"`` replays the earlier stage-release
scheme (through tile B's two S-ready barriers), which these checks reject.
"""
from __future__ import annotations

import random
from dataclasses import dataclass, field

LOCAL_CHUNKS = 8


class ProtocolError(AssertionError):
    pass


@dataclass
class Barrier:
    name: str
    expected: int
    pending: int = 0
    tx: int = 0
    completions: int = 0

    def __post_init__(self):
        self.pending = self.expected

    def _maybe_complete(self):
        if self.pending == 0 and self.tx == 0:
            self.completions += 1
            self.pending = self.expected

    def arrive(self, tx=0):
        if self.pending == 0:
            raise ProtocolError(f"over-arrival on {self.name} (phase {self.completions})")
        self.pending -= 1
        self.tx += tx
        self._maybe_complete()

    def complete_tx(self, nbytes):
        self.tx -= nbytes
        self._maybe_complete()

    def passes(self, parity):
        """Hardware try_wait.parity: true iff the current phase parity differs."""
        return (self.completions & 1) != parity


@dataclass
class State:
    n_chunks: int
    stages: int
    bars: dict = field(default_factory=dict)
    mma_queue: list = field(default_factory=list)   # issued, not completed (in order)
    tma_inflight: list = field(default_factory=list)
    mma_done: set = field(default_factory=set)       # ("S"|"PV", tile, chunk)
    stage_chunk: dict = field(default_factory=dict)  # stage -> chunk whose copy was issued
    stage_landed: dict = field(default_factory=dict)  # stage -> chunk whose copy landed
    p_stored: dict = field(default_factory=dict)     # (tile, chunk) -> warps that stored P
    pv_issued: set = field(default_factory=set)
    s_loaded: dict = field(default_factory=dict)     # chunk -> softmax warps that loaded S

    def bar(self, name):
        return self.bars[name]


def _wait(state, name, parity, completion):
    """A parity wait that stands for completion number `completion` of barrier `name`.

    Returns True when it passes; raises when it passes before that completion."""
    b = state.bar(name)
    if not b.passes(parity):
        return False
    if b.completions < completion + 1:
        raise ProtocolError(f"wait on {name} for completion {completion} passed at {b.completions}")
    return True


def producer(state, release):
    """Lane 0 of the producer warp (stencil_fwd.cu, ``warp == kProducerWarp``)."""
    k = state.stages
    for ch in range(state.n_chunks):
        s = ch % k
        if ch >= k:
            if release == "empty":
                while not _wait(state, f"empty{s}", (ch // k - 1) & 1, ch // k - 1):
                    yield ("wait", f"empty{s}")
            else:  # earlier scheme: tile B's S-ready barrier of S_B(x), x = ch - k + 2
                x = ch - k + 2
                while not _wait(state, f"sready1{x & 1}", (x >> 1) & 1, x >> 1):
                    yield ("wait", f"sready1{x & 1}")
        old = state.stage_chunk.get(s)
        if old is not None:
            for op in (("S", 0, old), ("S", 1, old), ("PV", 0, old), ("PV", 1, old)):
                if op not in state.mma_done:
                    raise ProtocolError(f"stage {s} overwritten with chunk {ch} while {op} is outstanding")
        state.bar(f"full{s}").arrive(tx=1)
        state.stage_chunk[s] = ch
        state.tma_inflight.append((s, ch))
        yield ("step", None)


def mma(state):
    """The MMA-issuing thread (``warp == kMmaWarp``)."""
    k, n = state.stages, state.n_chunks

    def commit(name):
        state.mma_queue.append(("commit", name))

    def issue_s(t, ch):
        s = ch % k
        if state.stage_landed.get(s) != ch:
            raise ProtocolError(f"S_{t}({ch}) reads stage {s} before chunk {ch} landed")
        if ch >= 2 and ("PV", t, ch - 2) not in state.mma_done:
            raise ProtocolError(f"S_{t}({ch}) overwrites P of chunk {ch - 2} before PV_{t}({ch - 2}) completed")
        state.mma_queue.append(("S", t, ch))
        commit(f"empty{(ch - 2) % k}" if (t == 1 and ch >= 2 and state.release == "empty")
               else f"sready{t}{ch & 1}")

    def waits(name, parity, completion):
        while not _wait(state, name, parity, completion):
            yield ("wait", name)

    yield from waits("qfull", 0, 0)
    for ch in range(2):
        yield from waits(f"full{ch % k}", (ch // k) & 1, ch // k)
        issue_s(0, ch)
        issue_s(1, ch)
        yield ("step", None)
    for c in range(n):
        ch = c + 2
        for t in range(2):   # PV_t(c), then (after it completed) S_t(c+2): tiles are decoupled
            yield from waits(f"pready{t}{c & 1}", (c >> 1) & 1, c >> 1)
            if len(state.p_stored.get((t, c), ())) != 4:
                raise ProtocolError(f"PV_{t}({c}) issued before all four warps stored P")
            state.mma_queue.append(("PV", t, c))
            state.pv_issued.add((t, c))
            commit(f"pvdone{t}{c & 1}")
            yield ("step", None)
            if ch >= n:
                continue
            if t == 0:
                yield from waits(f"full{ch % k}", (ch // k) & 1, ch // k)
            yield from waits(f"pvdone{t}{c & 1}", (c >> 1) & 1, c >> 1)
            issue_s(t, ch)
            yield ("step", None)
    commit("oready0")
    commit("oready1")
    commit("drain")
    yield from waits("drain", 0, 0)


def softmax(state, t, w, rng):
    """Softmax warp w of tile t (warps 0-7)."""
    k, n = state.stages, state.n_chunks

    def waits(name, parity, completion):
        while not _wait(state, name, parity, completion):
            yield ("wait", name)

    def pv_done(c):
        yield from waits(f"pvdone{t}{c & 1}", (c >> 1) & 1, c >> 1)
        if ("PV", t, c) not in state.mma_done:
            raise ProtocolError(f"O of tile {t} touched before PV_{t}({c}) completed")
        if (t, c + 1) in state.pv_issued:
            raise ProtocolError(f"O of tile {t} touched after PV_{t}({c + 1}) was issued")

    for ch in range(n):
        if ch == LOCAL_CHUNKS:
            yield from pv_done(LOCAL_CHUNKS - 1)
        if t == 1 and ch >= 2 and state.release == "empty":
            yield from waits(f"empty{(ch - 2) % k}", ((ch - 2) // k) & 1, (ch - 2) // k)
        else:
            yield from waits(f"sready{t}{ch & 1}", (ch >> 1) & 1, ch >> 1)
        if ("S", t, ch) not in state.mma_done:
            raise ProtocolError(f"S_{t}({ch}) read before it completed")
        yield ("step", None)
        state.p_stored.setdefault((t, ch), set()).add(w)
        if ch not in (0, LOCAL_CHUNKS) and rng.random() < 0.3:  # data-dependent rescale of O
            yield from pv_done(ch - 1)
        state.bar(f"pready{t}{ch & 1}").arrive()
        yield ("step", None)
    yield from waits(f"oready{t}", 0, 0)


def run(n_chunks=14, stages=4, seed=0, release="empty", max_steps=400000):
    """Replay one random interleaving; raises ProtocolError on a violation or deadlock."""
    rng = random.Random(seed)
    state = State(n_chunks=n_chunks, stages=stages)
    state.release = release
    bars = {"qfull": 1, "drain": 1, "oready0": 1, "oready1": 1}
    for s in range(4):
        bars[f"full{s}"] = 1
        bars[f"empty{s}"] = 1
    for t in range(2):
        for b in range(2):
            bars[f"sready{t}{b}"] = 1
            bars[f"pready{t}{b}"] = 4
            bars[f"pvdone{t}{b}"] = 1
    state.bars = {name: Barrier(name, cnt) for name, cnt in bars.items()}
    state.bar("qfull").arrive(tx=0)
    roles = {"producer": producer(state, release), "mma": mma(state)}
    for t in range(2):
        for w in range(4):
            roles[f"softmax{t}{w}"] = softmax(state, t, w, random.Random(rng.random()))
    return _schedule(state, roles, rng, max_steps)


def _next_completion(state, rng):
    """Index in the issue queue of the tensor-core operation that completes next.

    By default operations complete in issue order.  With ``state.ordered_by_acc`` (a map
    from operation kind to the accumulator it writes) only operations on the same
    accumulator keep their order, and a commit arrives once every operation issued before
    it has completed."""
    order = getattr(state, "ordered_by_acc", None)
    if order is None:
        return 0
    q, seen, ready = state.mma_queue, set(), []
    for i, op in enumerate(q):
        if op[0] == "commit":
            if all(o[0] == "commit" for o in q[:i]):
                ready.append(i)
            continue
        acc = order[op[0]](op)
        if acc not in seen:
            ready.append(i)
            seen.add(acc)
    return rng.choice(ready)


def _schedule(state, roles, rng, max_steps):
    """Run the role programs and asynchronous completions in a random order until all finish."""
    epoch = 0            # bumped whenever an asynchronous event changes some barrier
    blocked = {}         # role -> epoch of its last unsuccessful wait
    for _ in range(max_steps):
        events = ((["<copy lands>"] if state.tma_inflight else []) +
                  (["<tensor op completes>"] if state.mma_queue else []))
        if not roles and not events:
            return state
        live = [r for r in roles if blocked.get(r) != epoch]
        if not live and not events:
            raise ProtocolError(f"deadlock: {sorted(roles)} all wait")
        choice = rng.choice(live + events * 3)
        if choice == "<copy lands>":
            s, ch = state.tma_inflight.pop(rng.randrange(len(state.tma_inflight)))
            state.stage_landed[s] = ch
            state.bar(f"full{s}").complete_tx(1)
            epoch += 1
        elif choice == "<tensor op completes>":
            op = state.mma_queue.pop(_next_completion(state, rng))
            if op[0] == "commit":
                state.bar(op[1]).arrive()
            else:
                hook = getattr(state, "on_complete", None)
                if hook is not None:
                    hook(op)
                state.mma_done.add(op)
            epoch += 1
        else:
            try:
                kind, _ = next(roles[choice])
            except StopIteration:
                del roles[choice]
                blocked.pop(choice, None)
                epoch += 1
                continue
            if kind == "wait":
                blocked[choice] = epoch
            else:
                blocked.pop(choice, None)
                epoch += 1   # a role's step (an arrive, an issue) may unblock others
    raise ProtocolError(f"no progress after {max_steps} steps: roles left {sorted(roles)}")


# ----------------------------------------------------------------------------- dQ kernel
# Model of stencil_bwd_dq_kernel (pack3d_b200/csrc/stencil_bwd.cu): one 128-query tile per
# CTA with a single S buffer, a single dP buffer that receives dS, and the dQ accumulator;
# the ring's stages are released by the commit after dQ of the chunk they held.

def dq_producer(state):
    k = state.stages
    for ch in range(state.n_chunks):
        s = ch % k
        if ch >= k:
            while not _wait(state, f"empty{s}", (ch // k - 1) & 1, ch // k - 1):
                yield ("wait", f"empty{s}")
        old = state.stage_chunk.get(s)
        if old is not None:
            for op in [(kind, 0, old) for kind in ("S", "DP", "DQ")]:
                if op not in state.mma_done:
                    raise ProtocolError(f"stage {s} overwritten with chunk {ch} while {op} is outstanding")
        state.bar(f"full{s}").arrive(tx=1)
        state.stage_chunk[s] = ch
        state.tma_inflight.append((s, ch))
        yield ("step", None)


def dq_mma(state):
    k, n = state.stages, state.n_chunks

    def commit(name):
        state.mma_queue.append(("commit", name))

    def landed(c):
        if state.stage_landed.get(c % k) != c:
            raise ProtocolError(f"chunk {c} read before its copy landed")

    def issue_s(c):
        landed(c)
        if c >= 1 and len(state.s_read.get(c - 1, ())) != 4:
            raise ProtocolError(f"S({c}) overwrites S while the softmax may still read S({c - 1})")
        state.mma_queue.append(("S", 0, c))
        commit("sready")

    def issue_dp(c):
        landed(c)
        if c >= 1 and ("DQ", 0, c - 1) not in state.mma_done:
            raise ProtocolError(f"dP({c}) overwrites dS({c - 1}) before dQ({c - 1}) completed")
        state.mma_queue.append(("DP", 0, c))
        commit("dpready")

    def issue_dq(c):
        landed(c)
        if len(state.ds_stored.get(c, ())) != 4:
            raise ProtocolError(f"dQ({c}) issued before all four warps stored dS")
        state.mma_queue.append(("DQ", 0, c))
        state.dq_issued.add(c)
        commit("dqdone")

    def waits(name, completion):
        while not _wait(state, name, completion & 1, completion):
            yield ("wait", name)

    yield from waits("qfull", 0)
    yield from waits("full0", 0)
    issue_s(0)
    issue_dp(0)
    yield ("step", None)
    for c in range(n):
        more = c + 1 < n
        if more:
            yield from waits("sfree", c)
            yield from waits(f"full{(c + 1) % k}", (c + 1) // k)
            issue_s(c + 1)
            yield ("step", None)
        yield from waits("dsready", c)
        issue_dq(c)
        yield ("step", None)
        if not more:
            break
        yield from waits("dqdone", c)
        state.bar(f"empty{c % k}").arrive()   # dQ(c), the stage's last reader, completed
        issue_dp(c + 1)
        yield ("step", None)
    commit("drain")
    yield from waits("drain", 0)


def dq_softmax(state, w):
    n = state.n_chunks

    def waits(name, completion):
        while not _wait(state, name, completion & 1, completion):
            yield ("wait", name)

    for ch in range(n):
        if ch == LOCAL_CHUNKS:
            yield from waits("dqdone", LOCAL_CHUNKS - 1)
            if ("DQ", 0, LOCAL_CHUNKS - 1) not in state.mma_done or LOCAL_CHUNKS in state.dq_issued:
                raise ProtocolError("dQ_l read outside its window")
        yield from waits("sready", ch)
        if ("S", 0, ch) not in state.mma_done:
            raise ProtocolError(f"S({ch}) read before it completed")
        state.s_read.setdefault(ch, set()).add(w)
        state.bar("sfree").arrive()
        yield ("step", None)
        yield from waits("dpready", ch)
        if ("DP", 0, ch) not in state.mma_done:
            raise ProtocolError(f"dP({ch}) read before it completed")
        if ch >= 1 and ("DQ", 0, ch - 1) not in state.mma_done:
            raise ProtocolError(f"dS({ch}) overwrites dS({ch - 1}) while dQ({ch - 1}) may read it")
        state.ds_stored.setdefault(ch, set()).add(w)
        state.bar("dsready").arrive()
        yield ("step", None)
    yield from waits("dqdone", n - 1)
    if ("DQ", 0, n - 1) not in state.mma_done:
        raise ProtocolError("dQ read before the last product completed")


def run_dq(n_chunks=12, stages=3, seed=0, max_steps=400000):
    """Replay one random interleaving of the dQ kernel's protocol."""
    rng = random.Random(seed)
    state = State(n_chunks=n_chunks, stages=stages)
    state.ds_stored, state.dq_issued, state.s_read = {}, set(), {}
    # S, dP and dQ are three accumulators: only operations on the same one keep their order
    state.ordered_by_acc = {"S": lambda op: "s", "DP": lambda op: "dp", "DQ": lambda op: "dq"}
    bars = {"qfull": 1, "drain": 1, "sready": 1, "sfree": 4, "dpready": 1, "dsready": 4, "dqdone": 1}
    for s in range(4):
        bars[f"full{s}"] = 1
        bars[f"empty{s}"] = 1
    state.bars = {name: Barrier(name, cnt) for name, cnt in bars.items()}
    state.bar("qfull").arrive(tx=0)
    roles = {"producer": dq_producer(state), "mma": dq_mma(state)}
    for w in range(4):
        roles[f"softmax{w}"] = dq_softmax(state, w)
    return _schedule(state, roles, rng, max_steps)


# --------------------------------------------------------------- forward, one tile per CTA
# Model of the shipped stencil_fwd_kernel: one 128-row tile per CTA with a single S buffer
# and a separate P buffer in TMEM, four softmax warps (one per 32-row quarter).  S(c)
# commits to sfull; the softmax warps arrive on sfree once they have loaded S(c) into
# registers, and S(c + 1) may then overwrite it; they arrive on pfull once P(c) is stored;
# PV(c) commits to pfree (P buffer reusable, O quiet) and to empty[c % stages] (the ring
# stage of chunk c released to the producer).

def fwd1_producer(state):
    k = state.stages
    for ch in range(state.n_chunks):
        s = ch % k
        if ch >= k:
            while not _wait(state, f"empty{s}", (ch // k - 1) & 1, ch // k - 1):
                yield ("wait", f"empty{s}")
        old = state.stage_chunk.get(s)
        if old is not None:
            for op in (("S", 0, old), ("PV", 0, old)):
                if op not in state.mma_done:
                    raise ProtocolError(f"stage {s} overwritten with chunk {ch} while {op} is outstanding")
        state.bar(f"full{s}").arrive(tx=1)
        state.stage_chunk[s] = ch
        state.tma_inflight.append((s, ch))
        yield ("step", None)


def fwd1_mma(state, skip_sfree=False):
    k, n = state.stages, state.n_chunks

    def commit(name):
        state.mma_queue.append(("commit", name))

    def waits(name, completion):
        while not _wait(state, name, completion & 1, completion):
            yield ("wait", name)

    def issue_s(ch):
        if state.stage_landed.get(ch % k) != ch:
            raise ProtocolError(f"S({ch}) reads stage {ch % k} before chunk {ch} landed")
        if ch >= 1 and len(state.s_loaded.get(ch - 1, ())) != WARPS:
            raise ProtocolError(f"S({ch}) overwrites S({ch - 1}) before the softmax warps loaded it")
        state.mma_queue.append(("S", 0, ch))
        commit("sfull")

    yield from waits("qfull", 0)
    if n:
        yield from waits("full0", 0)
        issue_s(0)
        yield ("step", None)
    for c in range(n):
        if c + 1 < n:
            yield from waits(f"full{(c + 1) % k}", (c + 1) // k)
            if not skip_sfree:
                yield from waits("sfree", c)
            issue_s(c + 1)
            yield ("step", None)
        yield from waits(f"pfull{c % 2}", c // 2)     # one barrier per P buffer
        if len(state.p_stored.get((0, c), ())) != WARPS:
            raise ProtocolError(f"PV({c}) issued before all softmax warps stored P")
        state.mma_queue.append(("PV", 0, c))
        state.pv_issued.add((0, c))
        commit("pfree")
        commit(f"empty{c % k}")
        yield ("step", None)
    commit("oready")
    commit("drain")
    yield from waits("drain", 0)


WARPS = 4


def fwd1_softmax(state, w, rng, p_buffers=2, wait_on_rescale_only=False):
    """A softmax warp of the forward kernel.  P(c) goes to P buffer c % p_buffers; its last
    reader, PV(c - p_buffers), must have completed (with two buffers the kernel relies on the
    kSFull commit of S(c), issued after PV(c - 2)).  The warp waits for PV(c - 1) on every
    chunk (its O may be rescaled after that) except the global chunks of a warp on the
    fixed-reference path, which never rescale; the warp's path is drawn at random.
    ``wait_on_rescale_only`` is the broken variant that skips the wait unless it rescales."""
    n = state.n_chunks
    fixed = rng.random() < 0.5

    def waits(name, completion):
        while not _wait(state, name, completion & 1, completion):
            yield ("wait", name)

    def pv_done(c):
        yield from waits("pfree", c)
        if ("PV", 0, c) not in state.mma_done:
            raise ProtocolError(f"O touched before PV({c}) completed")
        if (0, c + 1) in state.pv_issued:
            raise ProtocolError(f"O touched after PV({c + 1}) was issued")

    for ch in range(n):
        if ch == LOCAL_CHUNKS:
            yield from pv_done(LOCAL_CHUNKS - 1)       # park the local output, free O
        yield from waits("sfull", ch)
        if ("S", 0, ch) not in state.mma_done:
            raise ProtocolError(f"S({ch}) read before it completed")
        if ("S", 0, ch + 1) in state.mma_done:
            raise ProtocolError(f"S({ch}) overwritten before this warp loaded it")
        state.s_loaded.setdefault(ch, set()).add(w)
        state.bar("sfree").arrive()
        yield ("step", None)
        local = ch < LOCAL_CHUNKS
        rescale = ch >= 1 and not (fixed and not local) and rng.random() < 0.3
        if ch >= 1 and (rescale if wait_on_rescale_only else not (fixed and not local)):
            yield from pv_done(ch - 1)
        if rescale:
            yield ("step", None)                       # a data-dependent rescale of O
        last_reader = ch - p_buffers
        if last_reader >= 0 and ("PV", 0, last_reader) not in state.mma_done:
            raise ProtocolError(f"P buffer {ch % p_buffers} overwritten while PV({last_reader}) may read it")
        state.p_stored.setdefault((0, ch), set()).add(w)
        state.bar(f"pfull{ch % 2}").arrive()
        yield ("step", None)
    yield from waits("oready", 0)
    if ("PV", 0, n - 1) not in state.mma_done:
        raise ProtocolError("O read before the last PV completed")


def run_fwd(n_chunks=14, stages=4, seed=0, max_steps=400000, skip_sfree=False, p_buffers=2,
            wait_on_rescale_only=False):
    """Replay one random interleaving of the (one-tile) forward kernel's protocol.

    Broken variants: ``skip_sfree`` (the MMA thread overwrites S without waiting for the
    softmax warps to load it), ``p_buffers=1`` (one P buffer, written without waiting for the
    PV that reads it on the fixed-reference global chunks) and ``wait_on_rescale_only`` (the
    kPFree waits skipped on every chunk without a rescale, which makes the parity waits that
    remain ambiguous)."""
    rng = random.Random(seed)
    state = State(n_chunks=n_chunks, stages=stages)
    state.ordered_by_acc = {"S": lambda op: "s", "PV": lambda op: "o"}  # S and O: separate accumulators
    bars = {"qfull": 1, "drain": 1, "oready": 1, "sfull": 1, "sfree": WARPS, "pfull0": WARPS, "pfull1": WARPS,
            "pfree": 1}
    for s in range(4):
        bars[f"full{s}"] = 1
        bars[f"empty{s}"] = 1
    state.bars = {name: Barrier(name, cnt) for name, cnt in bars.items()}
    state.bar("qfull").arrive(tx=0)
    roles = {"producer": fwd1_producer(state), "mma": fwd1_mma(state, skip_sfree)}
    for w in range(WARPS):
        roles[f"softmax{w}"] = fwd1_softmax(state, w, random.Random(rng.random()), p_buffers,
                                                wait_on_rescale_only)
    return _schedule(state, roles, rng, max_steps)


# ---------------------------------------------------- dK / dV kernels, two CTAs per SM
# Model of stencil_bwd_dkv_kernel and global_dkv_tc_kernel (pack3d_b200/csrc/stencil_bwd.cu):
# TMEM holds one S^T and one dP^T buffer; the softmax warps write dS^T back over dP^T as
# 16-bit pairs, and P^T either over S^T (``sep_p=False``) or into a buffer of its own
# (``sep_p=True``, head_dim <= 48).  S^T(c) commits sready, dP^T(c) dpready.  The warps load
# S^T(c) and arrive on sfree, exponentiate, wait for dpready(c), load dP^T(c), store P^T and
# dS^T and arrive on pdsready.  The MMA warp issues the products of chunk c after
# pdsready(c) (committing empty[c % stages] and accdone), waits for accdone(c) and issues
# dP^T(c + 1).  S^T(c + 1) is issued after sfree(c) with a separate P^T buffer, after
# accdone(c) otherwise.  Tensor-core operations complete in issue order only when they
# write the same accumulator (``ordered_by_acc``).  The model tracks each warp's TMEM
# regions (S, DP, P) and checks every read and overwrite against them.

def ip_producer(state):
    k = state.stages
    for ch in range(state.n_chunks):
        s = ch % k
        if ch >= k:
            while not _wait(state, f"empty{s}", (ch // k - 1) & 1, ch // k - 1):
                yield ("wait", f"empty{s}")
        old = state.stage_chunk.get(s)
        if old is not None:
            for op in (("S", 0, old), ("DP", 0, old), ("ACC", 0, old)):
                if op not in state.mma_done:
                    raise ProtocolError(f"stage {s} overwritten with chunk {ch} while {op} is outstanding")
            if len(state.read_vals.get(old, ())) != state.warps:
                raise ProtocolError(f"stage {s} overwritten while softmax warps may read chunk {old}'s lse")
        state.bar(f"full{s}").arrive(tx=1)  # expect_tx + copies
        state.stage_chunk[s] = ch
        state.tma_inflight.append((s, ch))
        yield ("step", None)
        state.bar(f"full{s}").arrive()      # lse / Delta stores of the warp
        yield ("step", None)


def ip_mma(state, skip_accdone=False):
    k, n, sep = state.stages, state.n_chunks, state.sep_p

    def commit(name):
        state.mma_queue.append(("commit", name))

    def landed(c):
        if state.stage_landed.get(c % k) != c:
            raise ProtocolError(f"chunk {c} read before its copy landed")

    def waits(name, completion):
        while not _wait(state, name, completion & 1, completion):
            yield ("wait", name)

    def issue(kind, c):
        landed(c)
        state.mma_queue.append((kind, 0, c))
        commit("sready" if kind == "S" else "dpready")

    yield from waits("kvfull", 0)
    yield from waits("full0", 0)
    issue("S", 0)
    issue("DP", 0)
    yield ("step", None)
    for c in range(n):
        if sep and c + 1 < n:
            yield from waits("sfree", c)
            yield from waits(f"full{(c + 1) % k}", (c + 1) // k)
            issue("S", c + 1)
            yield ("step", None)
        yield from waits("pdsready", c)
        landed(c)
        if len(state.pds_stored.get(c, ())) != state.warps:
            raise ProtocolError(f"dV/dK({c}) issued before all warps stored P/dS")
        state.mma_queue.append(("ACC", 0, c))
        commit(f"empty{c % k}")
        commit("accdone")
        yield ("step", None)
        if c + 1 < n:
            if not skip_accdone:
                yield from waits("accdone", c)
            if not sep:
                yield from waits(f"full{(c + 1) % k}", (c + 1) // k)
                issue("S", c + 1)
            issue("DP", c + 1)
            yield ("step", None)
    commit("accready")
    yield ("step", None)
    yield from waits("accready", 0)


def ip_softmax(state, w):
    n, sep = state.n_chunks, state.sep_p
    p_region = "P" if sep else "S"

    def waits(name, completion):
        while not _wait(state, name, completion & 1, completion):
            yield ("wait", name)

    def holds(region, want, what):
        got = state.tmem.get((w, region))
        if got != want:
            raise ProtocolError(f"warp {w} {what} but its TMEM lanes hold {got}")

    for ch in range(n):
        yield from waits("sready", ch)
        holds("S", ("S", ch), f"loaded S({ch})")
        if state.stage_chunk.get(ch % state.stages) != ch:
            raise ProtocolError(f"lse of chunk {ch} read from a stage holding another chunk")
        state.read_vals.setdefault(ch, set()).add(w)
        state.s_loaded.setdefault(ch, set()).add(w)
        state.bar("sfree").arrive()
        yield ("step", None)
        yield from waits("dpready", ch)
        holds("DP", ("DP", ch), f"loaded dP({ch})")
        yield ("step", None)
        old = state.tmem.get((w, p_region))
        if old is not None and old[0] == "P" and ("ACC", 0, old[1]) not in state.mma_done:
            raise ProtocolError(f"P({ch}) stored over P({old[1]}) before dV/dK({old[1]}) read it")
        state.tmem[(w, p_region)] = ("P", ch)
        state.tmem[(w, "DP")] = ("dS", ch)
        state.pds_stored.setdefault(ch, set()).add(w)
        state.bar("pdsready").arrive()
        yield ("step", None)
    yield from waits("accready", 0)
    if ("ACC", 0, n - 1) not in state.mma_done:
        raise ProtocolError("accumulators read before the last products completed")


def run_ip(n_chunks=10, stages=4, seed=0, warps=8, sep_p=True, skip_accdone=False, max_steps=400000):
    """Replay one random interleaving of the dK / dV kernels' protocol."""
    rng = random.Random(seed)
    state = State(n_chunks=n_chunks, stages=stages)
    state.pds_stored, state.read_vals, state.tmem, state.warps, state.sep_p = {}, {}, {}, warps, sep_p
    state.ordered_by_acc = {"S": lambda op: "s", "DP": lambda op: "dp", "ACC": lambda op: "acc"}
    bars = {"kvfull": 1, "accready": 1, "sready": 1, "sfree": warps, "dpready": 1, "pdsready": warps,
            "accdone": 1}
    for s in range(stages):
        bars[f"full{s}"] = 2
        bars[f"empty{s}"] = 1
    state.bars = {name: Barrier(name, cnt) for name, cnt in bars.items()}
    state.bar("kvfull").arrive(tx=0)
    roles = {"producer": ip_producer(state), "mma": ip_mma(state, skip_accdone)}
    for w in range(warps):
        roles[f"softmax{w}"] = ip_softmax(state, w)

    def on_complete(op):
        kind, _, c = op
        for v in range(warps):
            if kind == "S":
                held = state.tmem.get((v, "S"))
                if held is not None and held[0] == "S" and v not in state.s_loaded.get(held[1], ()):
                    raise ProtocolError(f"S({c}) overwrote S({held[1]}) before warp {v} loaded it")
                if held is not None and held[0] == "P" and ("ACC", 0, held[1]) not in state.mma_done:
                    raise ProtocolError(f"S({c}) overwrote P({held[1]}) before dV/dK({held[1]}) read it")
                state.tmem[(v, "S")] = ("S", c)
            elif kind == "DP":
                held = state.tmem.get((v, "DP"))
                if held is not None and held[0] == "dS" and ("ACC", 0, held[1]) not in state.mma_done:
                    raise ProtocolError(f"dP({c}) overwrote dS({held[1]}) before dV/dK({held[1]}) read it")
                state.tmem[(v, "DP")] = ("DP", c)
            elif kind == "ACC":
                p_held = state.tmem.get((v, "P" if state.sep_p else "S"))
                if p_held != ("P", c) or state.tmem.get((v, "DP")) != ("dS", c):
                    raise ProtocolError(f"dV/dK({c}) read lanes of warp {v} holding {p_held}, "
                                        f"{state.tmem.get((v, 'DP'))}")

    state.on_complete = on_complete
    return _schedule(state, roles, rng, max_steps)
