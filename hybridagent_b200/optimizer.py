"""Drop-in B200 replacement for HybridAgent's ``hybrid_rl.optimizer.ZeroOneAdamW``.

Same constructor, methods, public attributes, ownership and results as the reference
(hybrid_rl/optimizer.py:12-199); the work runs in ``libhybridagent_b200.so``:

=====================  =============================================  ==========================================
reference              what it does there                             here
=====================  =============================================  ==========================================
``__init__`` :13-86    greedy ownership, fp32 master/m/v per owned    same ownership; master/m/v live in one
                       tensor                                         packed fp32 buffer per dtype class, and at
                                                                      world > 1 the parameters are re-homed into
                                                                      an owner-major packed buffer
``all_reduce_grads``   used-mask MAX all-reduce; per owner, 64 Mi-    used-mask MAX (uint8, NCCL); one push kernel
:95-143                element bf16 buckets packed, ``dist.reduce``,  stores every gradient into its owner's receive
                       owner clones                                   buffer over NVLink; the owner's sum kernel adds
                                                                      the ranks' regions and emits the norm's square
                                                                      sums; owned grads are views of the sum
``clip_grad_norm``     per-tensor ``float().square().sum()``, fp32    the fused square sums (or one multi-tensor
:145-160               all-reduce, ``float(sqrt)``, bf16 ``mul_``     sum-of-squares kernel), one 8-byte NCCL
                                                                      all-reduce; the clip is folded into ``step``
``step`` :162-194      ~13 eager kernels per tensor, then one         one fused AdamW kernel per dtype class (28
                       ``dist.broadcast`` per tensor                  B/param for bf16) that also stores each new
                                                                      parameter into every peer's copy
=====================  =============================================  ==========================================

At world size > 1 the ranks map each other's packed buffers with CUDA IPC ("p2p" mode,
the default).  If any rank cannot map a peer, every rank uses "nccl" mode instead: a local
pack kernel, an NCCL reduce-scatter and an NCCL all-gather over the same buffers.  The
environment variable HYBRIDAGENT_B200_COMM=nccl selects that mode explicitly.

Numerics: every element is updated with the rounding torch's CUDA kernels give the
reference's op sequence, so master / exp_avg / exp_avg_sq and the parameter copy equal
the reference run on CUDA bit for bit.  The global norm is summed more accurately than
the reference's fp32 sum (fp64 partials), so it agrees to about 1e-7 relative; both are
rounded to fp32 before the square root as the reference does.  A non-finite gradient
makes the norm non-finite exactly where the reference's does.

Deliberate differences (documented surface):

* ``clip_grad_norm`` records the clip factor and ``step`` applies it while reading each
  gradient (same arithmetic as the reference's in-place ``grad.mul_``), so between the
  two calls -- and after ``step`` -- ``p.grad`` holds the unclipped values.  Call
  :meth:`apply_pending_clip` to scale the gradients in place instead.  A second
  ``clip_grad_norm`` or an ``all_reduce_grads`` before ``step`` applies it first, so
  chained calls see exactly the reference's values.
* At world_size > 1 ``param.data`` of every parameter is re-bound at construction to a
  view of the packed parameter buffer (each tensor takes its owner's values, as the
  reference's broadcast would) so the all-gather writes the model's weights in place;
  parameters must not be re-bound afterwards.
* At world_size > 1 in p2p mode the norm's square sums come out of ``all_reduce_grads``;
  ``clip_grad_norm`` recomputes them if an owned ``p.grad`` was replaced in between, but
  not if one was modified in place (the reference's trainer does neither).
* ``land_grads=True`` (new, opt-in, p2p mode) pushes the first two exchange rounds of each
  gradient to its owner while backward is still running (post-accumulate-grad hooks); results
  are unchanged: a gradient replaced, or modified in place through torch (its version counter
  moves), after its last landing is sent again whole by ``all_reduce_grads``.
* ``use_8bit=True`` (bitsandbytes PagedAdamW8bit, optimizer.py:76-86) is not provided.
* ``state_dict`` / ``load_state_dict`` are new (the reference has neither).
"""
from __future__ import annotations

import ctypes
import functools
import os
import weakref
from collections.abc import MutableMapping

import numpy as np
import torch

from . import _lib, layout
from ._lib import (HA_ADAMW_CHUNK, HA_BF16, HA_F16, HA_F32, HA_F64, HA_I32, HA_SUM_REGIONS_CHUNK, HA_SUMSQ_CHUNK,
                   HA_U8)

_CODES = {torch.float32: HA_F32, torch.bfloat16: HA_BF16, torch.float16: HA_F16}


def _nvtx(fn):
    """An NVTX range named ZeroOneAdamW.<method> around each call."""
    name = f"ZeroOneAdamW.{fn.__name__}"

    @functools.wraps(fn)
    def wrapper(*args, **kwargs):
        torch.cuda.nvtx.range_push(name)
        try:
            return fn(*args, **kwargs)
        finally:
            torch.cuda.nvtx.range_pop()
    return wrapper
_TORCH = {v: k for k, v in _CODES.items()}
STATE_FORMAT = "hybridagent_b200.zero1_adamw/1"


class _Table:
    """A host table (numpy structured array) mirrored in device memory.

    ``upload()`` copies the current host contents through one of a small ring of pinned
    buffers, so rewriting the table never waits for the GPU to consume an earlier copy
    (a ring slot is reused only after its previous copy has completed)."""

    RING = 3

    def __init__(self, n: int, dtype: np.dtype, device: torch.device):
        self.np = np.zeros(max(n, 1), dtype=dtype)
        nbytes = self.np.nbytes
        self.dev = torch.empty(nbytes, dtype=torch.uint8, device=device)
        self._ring = [torch.empty(nbytes, dtype=torch.uint8, pin_memory=True) for _ in range(self.RING)]
        self._events: list[torch.cuda.Event | None] = [None] * self.RING
        self._next = 0

    def upload(self) -> None:
        k = self._next
        self._next = (k + 1) % self.RING
        if self._events[k] is not None:
            self._events[k].synchronize()
        buf = self._ring[k]
        np.copyto(buf.numpy(), self.np.view(np.uint8))
        self.dev.copy_(buf, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        self._events[k] = ev

    @property
    def ptr(self) -> int:
        return self.dev.data_ptr()


class _ParamSteps(MutableMapping):
    """``param_steps`` of the reference (index -> per-tensor step count) backed by an array."""

    def __init__(self, counts: np.ndarray, owned: list[int]):
        self._counts = counts
        self._owned = set(owned)
        self._order = list(owned)
        self.version = 0

    def __getitem__(self, i: int) -> int:
        if i not in self._owned:
            raise KeyError(i)
        return int(self._counts[i])

    def __setitem__(self, i: int, v: int) -> None:
        if i not in self._owned:
            raise KeyError(f"tensor {i} is not owned by this rank")
        self._counts[i] = int(v)
        self.version += 1  # tables staged with the old counts are stale

    def __delitem__(self, i: int) -> None:
        raise TypeError("param_steps entries cannot be removed")

    def __iter__(self):
        return iter(self._order)

    def __len__(self) -> int:
        return len(self._order)

    def __repr__(self) -> str:
        return repr(dict(self.items()))


class _Class:
    """Device state of one dtype class on this rank."""

    def __init__(self, opt: "ZeroOneAdamW", cls: layout.DtypeClass):
        self.code = cls.code
        self.dtype = _TORCH[cls.code]
        self.layout = cls
        self.owned = cls.owned(opt.owner, opt.rank)
        dev = opt.device
        W, r = opt.world, opt.rank
        numel = opt._numels
        # --- packed parameters and the gradient receive window (world > 1), IPC-shareable;
        # the reduced-gradient buffer depends on the mode (set_mode)
        self.packed_param = None
        if W > 1:
            from .p2p import DeviceBuffer
            self.param_buf = DeviceBuffer(W * cls.seg_len, self.dtype, dev)
            self.packed_param = self.param_buf.tensor
            esz = self.packed_param.element_size()
            budget = int(os.environ.get("HYBRIDAGENT_B200_RECV_BYTES", str(4 << 30)))
            self.round_elems = layout.round_elems_for(cls, W, esz, budget)
            self.recv_buf = DeviceBuffer(2 * W * self.round_elems, self.dtype, dev)
            for i in cls.indices:
                p = opt.params[i]
                start = opt.owner[i] * cls.seg_len + cls.offset[i]
                slot = self.packed_param[start:start + numel[i]].view(p.shape)
                slot.copy_(p.data)
                p.data = slot
        # --- fp32 state of the owned tensors
        own_len = max(cls.own_len[r], layout.ALIGN)
        self.exp_avg_buf = torch.zeros(own_len, dtype=torch.float32, device=dev)
        self.exp_avg_sq_buf = torch.zeros(own_len, dtype=torch.float32, device=dev)
        self.master_buf = None if self.code == HA_F32 else torch.empty(own_len, dtype=torch.float32, device=dev)
        for i in self.owned:
            p = opt.params[i]
            o = cls.offset[i]
            opt.exp_avg[i] = self.exp_avg_buf[o:o + numel[i]].view(p.shape)
            opt.exp_avg_sq[i] = self.exp_avg_sq_buf[o:o + numel[i]].view(p.shape)
            if self.code == HA_F32:
                opt.master[i] = p.data  # optimizer.py:71-73: the fp32 parameter is the master
                opt.master_is_parameter[i] = True
            else:
                opt.master[i] = self.master_buf[o:o + numel[i]].view(p.shape)
                opt.master[i].copy_(p.data)  # float() of the parameter
                opt.master_is_parameter[i] = False
        # --- device tables
        self.table = _Table(len(self.owned), _lib.TENSOR_DTYPE, dev)
        tab = self.table.np
        for k, i in enumerate(self.owned):
            tab[k]["master"] = opt.master[i].data_ptr()
            tab[k]["exp_avg"] = opt.exp_avg[i].data_ptr()
            tab[k]["exp_avg_sq"] = opt.exp_avg_sq[i].data_ptr()
            tab[k]["param"] = 0 if self.code == HA_F32 else opt.params[i].data_ptr()
            tab[k]["numel"] = numel[i]
        owned_numels = [numel[i] for i in self.owned]
        self.lrs = np.ascontiguousarray([opt.lrs[i] for i in self.owned], dtype=np.float64)
        self.adamw_chunks = self._device_chunks(owned_numels, HA_ADAMW_CHUNK, dev)
        self.sumsq_chunks = self._device_chunks(owned_numels, HA_SUMSQ_CHUNK, dev)
        self.partials = torch.empty(max(self.sumsq_chunks[1], 1), dtype=torch.float64, device=dev)
        self.move = None
        self.peers = _lib.Peers()
        # changed-groups-only writes: the groups stored by the last such update (device counter,
        # read back without waiting) decide whether the next update is one too
        self.changed_dev = torch.zeros(1, dtype=torch.int64, device=dev)
        self.changed_host = torch.zeros(1, dtype=torch.int64, pin_memory=True)
        self.changed_event: torch.cuda.Event | None = None
        self.delta_next = True
        self.full_run = 0  # consecutive full updates chosen by the count (a changed-groups one is tried after 8)
        self.last_changed: int | None = None
        self.groups = sum((numel[i] + 3) // 4 for i in self.owned)  # 4-element groups owned

    def set_mode(self, opt: "ZeroOneAdamW", recv_bases: list[int] | None, param_bases: list[int] | None) -> None:
        """p2p (peers' receive windows and parameter buffers mapped) or the local nccl pack.

        p2p: this rank's gradients move to their owners in rounds (layout.exchange_pieces):
        round k covers elements [bounds[k], bounds[k+1]) of every owner's segment (k*S, unless
        the last round is split) and lands in half k % 2 of the owner's double-buffered receive
        window, region <this rank> of S elements; the owner adds the regions into ``own_grad``.  nccl: the whole owner-major pack of W segments
        is reduce-scattered in place."""
        cls, W, r, dev = self.layout, opt.world, opt.rank, opt.device
        numel = opt._numels
        esz = self.packed_param.element_size()
        if recv_bases is not None:
            S = self.round_elems
            pc = layout.exchange_pieces(cls, opt.owner, numel, S, opt.tail_split)
            self.pieces = pc
            self.own_grad = torch.zeros(max(cls.own_len[r], layout.ALIGN), dtype=self.dtype, device=dev)
            base = self.own_grad
            own0 = 0
            self.move = _Table(len(pc.count), _lib.COPY_DTYPE, dev)
            dst = layout.piece_destinations(pc, recv_bases, r, W, esz)
            self.piece_dst = dst
            self.move.np["dst"][:len(dst)] = dst
            self.move.np["numel"][:len(dst)] = pc.count
            self.piece_src_bytes = (pc.src_off * esz).astype(np.uint64)
            # per round: the push's chunk list (every piece; or, with the copy-engine push, this
            # rank's own pieces only) and the copy-engine groups of the pieces bound for peers
            self.round_chunks, self.round_remote = [], []
            for k in range(pc.n_rounds):
                entries, groups = layout.round_push_split(pc, k, r, opt.push_streams, opt.push_kernel_share, W)
                self.round_remote.append(groups)
                tab = layout.interleaved_chunks(entries, pc.owner, pc.count, r, W, HA_ADAMW_CHUNK)
                _lib.call("ha_check_chunks", len(pc.count), _lib.np_ptr(np.ascontiguousarray(pc.count)),
                          _lib.np_ptr(tab), len(tab), HA_ADAMW_CHUNK)
                self.round_chunks.append((torch.from_numpy(tab.view(np.uint8).copy()).to(dev) if len(tab) else None,
                                          len(tab)))
            self.own_counts = pc.own_counts(cls, r)
            # gradient landing: the pieces that may be pushed during backward (rounds 0 and 1)
            self.land_pieces = layout.landing_pieces(pc, len(cls.indices))
            self.land_mask = (pc.round < layout.LAND_ROUNDS) & (pc.tensor >= 0)
            n_part = max(-(-S // HA_SUM_REGIONS_CHUNK), 1)
            # one buffer serves every round: the sums run one after another on one stream
            self.region_partials = torch.empty(n_part, dtype=torch.float64, device=dev)
            self.peers = _lib.Peers()
            deltas = layout.peer_deltas(param_bases, r)
            for q, d in enumerate(deltas):
                self.peers.delta[q] = d
            self.peers.n = len(deltas)
            # copy-engine all-gather: per part of the update, one copy per peer of the part's
            # elements of this rank's segment to the same place in the peer's buffer
            self.gather_parts, self.gather_copies = [], []
            if opt.gather_mode == "ce" and self.adamw_chunks[1]:
                tab = layout.chunk_table([numel[i] for i in self.owned], HA_ADAMW_CHUNK)
                self.gather_parts = layout.gather_parts(tab, [cls.offset[i] for i in self.owned],
                                                        [numel[i] for i in self.owned], HA_ADAMW_CHUNK,
                                                        max(opt.gather_part_bytes // esz, HA_ADAMW_CHUNK))
                seg = param_bases[r] + r * cls.seg_len * esz
                for _, _, e0, e1 in self.gather_parts:
                    per_peer = []
                    for j in range(W - 1):  # peer (r + 1 + j) % W first: every peer's ingress busy at once
                        q = (r + 1 + j) % W
                        cp = np.zeros(1, dtype=_lib.COPY_DTYPE)
                        cp["src"] = seg + e0 * esz
                        cp["dst"] = param_bases[q] - param_bases[r] + seg + e0 * esz
                        cp["numel"] = e1 - e0
                        per_peer.append(cp)
                    self.gather_copies.append(per_peer)
        else:
            self.recv_buf = None  # not used without peer mappings
            self.grad_buf = torch.zeros(W * cls.seg_len, dtype=self.dtype, device=dev)
            base = self.grad_buf
            own0 = r * cls.seg_len
            self.move = _Table(len(cls.indices), _lib.COPY_DTYPE, dev)
            dst = layout.push_destinations(cls, opt.owner, r, esz, None, self.grad_buf.data_ptr())
            self.move.np["dst"][:len(dst)] = dst
            self.move.np["numel"][:len(dst)] = [numel[i] for i in cls.indices]
            self.move_chunks = self._device_chunks([numel[i] for i in cls.indices], HA_ADAMW_CHUNK, dev)
        # reduced gradients handed to the caller as p.grad (optimizer.py:141)
        self.grad_view = {i: base[own0 + cls.offset[i]:own0 + cls.offset[i] + numel[i]].view(opt.params[i].shape)
                          for i in self.owned}

    @staticmethod
    def _device_chunks(numels: list[int], chunk: int, dev) -> tuple[torch.Tensor | None, int]:
        tab = layout.chunk_table(numels, chunk)
        if len(tab) == 0:
            return None, 0
        t = torch.from_numpy(tab.view(np.uint8).copy()).to(dev)
        return t, len(tab)


class ZeroOneAdamW:
    """ZeRO-1 AdamW over CUDA parameters (drop-in for hybrid_rl.optimizer.ZeroOneAdamW)."""

    def __init__(self, param_groups, *, rank: int, world_size: int, betas=(0.9, 0.999), eps: float = 1e-8,
                 weight_decay: float = 0.0, use_8bit: bool = False, comm_timeout_s: float | None = None,
                 land_grads: bool = False):
        # argument handling and errors as optimizer.py:24-44; comm_timeout_s (world > 1): seconds a
        # collective may wait for the other ranks before the communicator is aborted and the call
        # raises CommFailure (default HYBRIDAGENT_B200_COMM_TIMEOUT_S or 1800); land_grads: while
        # backward is still running, push gradients to their owners (world > 1, p2p mode) or take
        # the norm's square sums (world 1)
        self.rank = int(rank)
        self.world = int(world_size)
        self.betas = tuple(float(value) for value in betas)
        self.eps = float(eps)
        self.weight_decay = float(weight_decay)
        self.use_8bit = bool(use_8bit)
        if len(self.betas) != 2 or any(not 0.0 <= value < 1.0 for value in self.betas):
            raise ValueError("betas must contain two values in [0, 1)")
        if self.world < 1 or not 0 <= self.rank < self.world:
            raise ValueError(f"invalid rank/world {self.rank}/{self.world}")
        self.step_count = 0
        flat: list[tuple[torch.nn.Parameter, float]] = []
        seen: set[int] = set()
        for group in param_groups:
            for parameter in group["params"]:
                if parameter.requires_grad and id(parameter) not in seen:
                    seen.add(id(parameter))
                    flat.append((parameter, float(group["lr"])))
        if not flat:
            raise ValueError("ZeroOneAdamW received no trainable parameters")
        if self.use_8bit:
            raise NotImplementedError("use_8bit (bitsandbytes PagedAdamW8bit) is not provided by hybridagent_b200")
        self.params = [p for p, _ in flat]
        self.lrs = [lr for _, lr in flat]
        self.device = self.params[0].device
        if self.device.type != "cuda":
            raise RuntimeError(f"hybridagent_b200.ZeroOneAdamW runs on CUDA devices only; parameters are on "
                               f"{self.device} (there is no CPU path)")
        for p in self.params:
            if p.device != self.device:
                raise RuntimeError(f"all parameters must be on one device: {p.device} vs {self.device}")
            if p.dtype not in _CODES:
                raise TypeError(f"unsupported parameter dtype {p.dtype}")
            if not p.is_contiguous():
                raise ValueError("parameters must be contiguous")
        _lib.lib()  # fail loudly now if the CUDA library is missing
        self._numels = [p.numel() for p in self.params]
        with torch.cuda.device(self.device):
            self._plan = layout.plan(self._numels, [_CODES[p.dtype] for p in self.params], self.world)
            self.owner = list(self._plan.owner)
            self.master: dict[int, torch.Tensor] = {}
            self.master_is_parameter: dict[int, bool] = {}
            self.exp_avg: dict[int, torch.Tensor] = {}
            self.exp_avg_sq: dict[int, torch.Tensor] = {}
            self._steps = np.zeros(len(self.params), dtype=np.int64)
            self._table_epoch = 0  # table uploads so far (a staged table is valid while it is the last)
            self._staged = None
            owned_all = [i for i in range(len(self.params)) if self.owner[i] == self.rank]
            self.param_steps = _ParamSteps(self._steps, owned_all)
            self.owned_numel = sum(self._numels[i] for i in owned_all)
            self._comm = None
            self._peer_map = None
            self.comm_mode = "local"
            self.gather_mode = "kernel"
            self._gather_streams: list = []
            if self.world > 1:
                from .comm import NcclComm
                self._comm = NcclComm(self.rank, self.world, timeout_s=comm_timeout_s)
            self._classes = [_Class(self, c) for c in self._plan.classes]
            self._norm_buf = torch.zeros(len(self._classes), dtype=torch.float64, device=self.device)
            # world > 1: one all-reduce(max) of [used(T), dirty(T)] (see _detect_dirty)
            self._used_dev = torch.zeros(2 * len(self.params), dtype=torch.uint8, device=self.device)
            self._barrier_buf = torch.zeros(1, dtype=torch.int32, device=self.device)
            # pinned landing buffers of the host reads (deadline-aware waits at world > 1)
            self._norm_host = torch.zeros(len(self._classes), dtype=torch.float64, pin_memory=True)
            if self.world > 1:
                # this rank's mask (uploaded asynchronously: the next call rewrites it only after
                # reading the all-reduce that follows the upload) and the all-reduced mask
                self._used_local = torch.zeros(2 * len(self.params), dtype=torch.uint8, pin_memory=True)
                self._used_host = torch.zeros(2 * len(self.params), dtype=torch.uint8, pin_memory=True)
                self._setup_world()
            torch.cuda.current_stream().synchronize()
        # changed-groups-only parameter writes (ha_adamw_step_delta) need every copy of a parameter
        # to hold RNE(master) on entry.  Torch's version counters tell when anything else wrote a
        # parameter or a master; such tensors are "dirty" (the same set on every rank) and the
        # next step writes every parameter in full, as the reference does.
        self.delta_writes = os.environ.get("HYBRIDAGENT_B200_DELTA", "1") != "0"
        # above this fraction of changed groups (last update) the next update writes in full: with
        # most groups changing, scattered stores cost more than a full one (measured on B200 at one
        # GPU: 0.5 % changed -> 6 % faster than the full write, ~90 % changed -> 29 % slower)
        self.delta_max_fraction = float(os.environ.get("HYBRIDAGENT_B200_DELTA_MAX_FRACTION",
                                                       "0.05" if self.world == 1 else "0.1"))

        self._dirty = np.zeros(len(self.params), dtype=bool)
        self._force_dirty = np.zeros(len(self.params), dtype=bool)
        self._seen_params = self._param_versions()
        self._seen_masters = self._master_versions()
        self._dense_this_step = True
        self._last_used: np.ndarray | None = None  # world > 1: the used set of the last all_reduce_grads
        self.dense_steps = 0  # steps that wrote every parameter (delta off, fp32 classes aside)
        self._pending_clip: float | None = None
        self._fused_sumsq: list | None = None
        self._grad_cache: dict[int, tuple] = {}
        self.timer = None  # optional phase timer: .begin(name) / .end(name) around kernel launches
        self.launches = 0  # kernels of libhybridagent_b200 launched so far
        self.landing_enabled = False  # gradient landing active (toggle it off for non-final backward passes)
        self.land_launches = 0  # early pushes launched from the landing hooks
        self._land_hooks: list = []
        self._landed: dict[int, tuple[torch.Tensor, int]] = {}  # index -> (gradient, its version when pushed)
        self._lland = False  # world 1: square sums taken as gradients land (_setup_landing_local)
        self.land_norm_steps = 0  # clip_grad_norm calls served by those sums
        if land_grads and self.comm_mode == "p2p":
            self._setup_landing()
        elif land_grads and self.world == 1:
            self._setup_landing_local()

    def _setup_world(self) -> None:
        """Owners' parameter values to every rank (the reference's broadcast), then the
        peer mappings (p2p) or the nccl fallback, chosen identically on every rank."""
        for c in self._classes:
            own = c.packed_param.data_ptr() + self.rank * c.layout.seg_len * c.packed_param.element_size()
            self._comm.all_gather(own, c.packed_param.data_ptr(), c.layout.seg_len, c.code)
        # HYBRIDAGENT_B200_PUSH_STREAMS=N > 0: the pieces bound for peers go to the copy engines
        # on N streams, and the SMs only copy this rank's own pieces and sum.  Measured on B200 at
        # world 2 (Qwen3-8B set): 33.0 ms per step against 36.2 with the kernel push, whose remote
        # stores need nearly every SM and starve the owner sums; the copy engines move 669 GB/s.
        # At world > 2 this rank's own share and the sums shrink as 1/W: the kernel push stays.
        push = os.environ.get("HYBRIDAGENT_B200_PUSH_STREAMS", "2" if self.world == 2 else "0")
        self.push_streams = -1 if push == "peer" else int(push)  # "peer": one copy-engine stream per peer
        # with the copy-engine push: the share of the peer-bound bytes (smallest pieces first) that
        # the push kernel stores instead, using SM time the local copies and sums leave idle and
        # link bandwidth the copy engines leave unused (world 2: 0.1 -> 32.4 ms, 0 -> 33.0, 0.2 -> 32.7)
        self.push_kernel_share = float(os.environ.get("HYBRIDAGENT_B200_PUSH_KERNEL_SHARE", "0.1"))
        # the push kernel's grid: 0 -- one CTA per 16384-element chunk (every SM busy pushing);
        # N > 0 -- N CTAs walking the round's chunk list, each with 4 vectors per thread in
        # flight, leaving the other SM slots to the owner sums of the previous round.  Measured
        # on B200 at world 2 (kernel push of every piece): one CTA per chunk 34.4 ms per step (the
        # starved sums of the last rounds stay exposed), 148 CTAs 32.1, 296 31.1, 592 31.0.  With
        # the copy-engine push the kernel only copies this rank's own pieces: one CTA per chunk
        sms = torch.cuda.get_device_properties(self.device).multi_processor_count
        self.push_ctas = int(os.environ.get("HYBRIDAGENT_B200_PUSH_CTAS", str(4 * sms if self.push_streams == 0 else 0)))
        # the parameter all-gather (p2p): "kernel" -- the update kernel stores every new value into
        # every peer's copy; "ce" -- the update runs in parts of HYBRIDAGENT_B200_GATHER_PART_BYTES and
        # the copy engines send each finished part to every peer (one stream per peer) while the
        # next part updates, so the SMs issue no remote store
        self.gather_mode = os.environ.get("HYBRIDAGENT_B200_GATHER", "kernel")
        if self.gather_mode not in ("kernel", "ce"):
            raise ValueError(f"HYBRIDAGENT_B200_GATHER={self.gather_mode!r}: expected kernel or ce")
        self.gather_part_bytes = int(os.environ.get("HYBRIDAGENT_B200_GATHER_PART_BYTES", str(128 << 20)))
        # the last exchange round cut into up to this many more rounds of halving length
        # (layout.round_bounds): the owner sum after the last push is the one nothing overlaps
        self.tail_split = int(os.environ.get("HYBRIDAGENT_B200_TAIL_SPLIT", "0"))
        if self.tail_split < 0:
            raise ValueError(f"HYBRIDAGENT_B200_TAIL_SPLIT={self.tail_split}: expected >= 0")
        want = os.environ.get("HYBRIDAGENT_B200_COMM", "p2p")
        if want not in ("p2p", "nccl"):
            raise ValueError(f"HYBRIDAGENT_B200_COMM={want!r}: expected p2p or nccl")
        ok = 0
        if want == "p2p":
            from .p2p import PeerMap
            bufs = {}
            for k, c in enumerate(self._classes):
                bufs[f"recv{k}"] = c.recv_buf
                bufs[f"param{k}"] = c.param_buf
            self._peer_map = PeerMap(bufs, self.rank, self.world)
            ok = 1 if self._peer_map.ok else 0
        flag = torch.tensor([1 - ok], dtype=torch.int32, device=self.device)
        self._comm.all_reduce_max(flag, HA_I32)  # every rank takes the same mode
        use_p2p = int(self._comm.read(flag, torch.zeros(1, dtype=torch.int32, pin_memory=True),
                                      "all-reduce(max) of the p2p flag")[0]) == 0
        if not use_p2p and self._peer_map is not None:
            self._peer_map.close()
            self._peer_map = None
        self.comm_mode = "p2p" if use_p2p else "nccl"
        for k, c in enumerate(self._classes):
            if use_p2p:
                c.set_mode(self, self._peer_map.bases[f"recv{k}"], self._peer_map.bases[f"param{k}"])
            else:
                c.set_mode(self, None, None)
            c.move.upload()
        self._sum_stream = torch.cuda.Stream(device=self.device) if use_p2p else None
        n_push = self.world - 1 if self.push_streams < 0 else self.push_streams
        self._push_streams = [torch.cuda.Stream(device=self.device) for _ in range(n_push)] if use_p2p else []
        self._gather_streams = ([torch.cuda.Stream(device=self.device) for _ in range(self.world - 1)]
                                if use_p2p and self.gather_mode == "ce" else [])
        rounds = max(c.pieces.n_rounds for c in self._classes) if use_p2p else 1
        self._norm_rounds = torch.zeros((len(self._classes), rounds), dtype=torch.float64, device=self.device)
        self._norm_rounds_host = torch.zeros((len(self._classes), rounds), dtype=torch.float64, pin_memory=True)

    def _exchange_rounds(self) -> None:
        """p2p gradient exchange: per round, every rank pushes its pieces into the owners'
        receive windows, one barrier, then each owner adds the regions of that round into
        its reduced gradients and the norm's square sums.

        The sums run on a second stream so round k's sum (HBM) overlaps round k+1's push
        (NVLink).  The window is double-buffered (half k % 2): barrier k+1 is enqueued only
        after this rank's sum k has finished, so when barrier k+1 completes every owner has
        read half k % 2 and round k+2 may overwrite it; sum k waits for barrier k, so it reads
        only after every rank's round-k pushes landed."""
        main = torch.cuda.current_stream()
        side = self._sum_stream
        rounds = max(c.pieces.n_rounds for c in self._classes)
        summed = None  # event after the previous round's sums on the side stream
        for k in range(rounds):
            self._phase("push", True)
            if self._push_streams:  # pieces bound for peers: copy engines, one group per stream
                ready = torch.cuda.Event()
                ready.record(main)  # after the tables, the used mask and barrier k-1
                for j, st in enumerate(self._push_streams):
                    st.wait_event(ready)
                    for c in self._classes:
                        if k < c.pieces.n_rounds and len(c.round_remote[k][j]):
                            copies = c.move.np[c.round_remote[k][j]]
                            _lib.call("ha_copy_async", _lib.np_ptr(copies), len(copies),
                                      c.packed_param.element_size(), st.cuda_stream)
            for c in self._classes:
                if k < c.pieces.n_rounds and c.round_chunks[k][1]:
                    ch, n = c.round_chunks[k]
                    if self.push_ctas > 0:
                        _lib.call("ha_gather_capped", c.move.ptr, ch.data_ptr(), n, HA_ADAMW_CHUNK,
                                  c.packed_param.element_size(), self.push_ctas, main.cuda_stream)
                    else:
                        _lib.call("ha_gather", c.move.ptr, ch.data_ptr(), n, HA_ADAMW_CHUNK,
                                  c.packed_param.element_size(), main.cuda_stream)
                    self.launches += 1
            for st in self._push_streams:
                main.wait_stream(st)
            self._phase("push", False)
            if summed is not None:
                main.wait_event(summed)  # this rank has read the half that round k+1 rewrites
            self._phase("barrier", True)
            self._barrier()  # every rank's pushes of round k have landed
            self._phase("barrier", False)
            landed = torch.cuda.Event()
            landed.record(main)
            side.wait_event(landed)
            with torch.cuda.stream(side):
                self._phase("sum_regions", True)
                for ci, c in enumerate(self._classes):
                    if k >= c.pieces.n_rounds:
                        continue
                    S, esz = c.round_elems, c.packed_param.element_size()
                    count = c.own_counts[k]
                    window = c.recv_buf.ptr + (k % 2) * self.world * S * esz
                    own = c.own_grad.data_ptr() + int(c.pieces.bounds[k]) * esz
                    _lib.call("ha_sum_regions", window, self.world, S, count, own,
                              c.code, c.region_partials.data_ptr(), self._norm_rounds[ci, k:].data_ptr(),
                              side.cuda_stream)
                    self.launches += 2 if count else 1
                self._phase("sum_regions", False)
            summed = torch.cuda.Event()
            summed.record(side)
        main.wait_event(summed)  # the reduced gradients and square sums are complete for later work

    def _barrier(self) -> None:
        """Stream-ordered barrier across ranks: returns on every rank's stream only after every
        rank's earlier work (this rank's peer stores included) has completed."""
        self._comm.all_reduce_sum(self._barrier_buf, HA_I32)

    # ---------------------------------------------------------------- dirty tracking
    def _param_versions(self) -> np.ndarray:
        """(address, torch version) of every parameter: a re-bound or in-place-modified
        parameter shows up as a change."""
        out = np.zeros((len(self.params), 2), dtype=np.int64)
        for i, p in enumerate(self.params):
            out[i, 0] = p.data_ptr()
            out[i, 1] = p._version
        return out

    def _master_versions(self) -> list[int]:
        """Torch version of each class's packed master buffer (the masters are views of it, so
        an in-place write to any of them moves it); -1 for fp32 classes (master = parameter)."""
        return [-1 if c.master_buf is None else c.master_buf._version for c in self._classes]

    def _detect_dirty(self) -> np.ndarray:
        """Tensors whose parameter (any rank's copy) or master was written by anything other than
        this optimizer's kernels since the versions were last recorded, plus those marked with
        mark_parameters_dirty(); records the current versions."""
        now = self._param_versions()
        dirty = (now != self._seen_params).any(axis=1) | self._force_dirty
        masters = self._master_versions()
        for c, was, is_ in zip(self._classes, self._seen_masters, masters):
            if was != is_:
                dirty[c.owned] = True
        self._seen_params, self._seen_masters = now, masters
        self._force_dirty[:] = False
        return dirty

    def mark_parameters_dirty(self, indices=None) -> None:
        """Declares parameters (all, or the given flat indices) as written outside torch's
        in-place ops -- through ``.data`` or a raw pointer -- so the next step writes them in
        full on every rank, as the reference's broadcast would.  In-place torch writes
        (``p.copy_``, a model's ``load_state_dict``, ``optimizer.master[i].copy_``) are detected
        without it.  At world size > 1 call it before ``all_reduce_grads``."""
        if indices is None:
            self._force_dirty[:] = True
        else:
            self._force_dirty[np.asarray(list(indices), dtype=np.int64)] = True

    # ---------------------------------------------------------------- helpers
    def _phase(self, name: str, start: bool) -> None:
        """Marks a phase: an NVTX range (Nsight timelines) and, if a timer is attached, its
        CUDA events."""
        if start:
            torch.cuda.nvtx.range_push(f"ZeroOneAdamW.{name}")
        else:
            torch.cuda.nvtx.range_pop()
        if self.timer is not None:
            (self.timer.begin if start else self.timer.end)(name)

    @staticmethod
    def _stream() -> int:
        return torch.cuda.current_stream().cuda_stream

    def _owned_grads(self, c: _Class) -> tuple[list[torch.Tensor | None], np.ndarray]:
        grads, ptrs = [], np.zeros(len(c.owned), dtype=np.uint64)
        for k, i in enumerate(c.owned):
            g = self.params[i].grad
            if g is not None:
                if g.dtype != c.dtype or g.numel() != self._numels[i] or g.device != self.device:
                    raise RuntimeError(f"gradient of tensor {i} has dtype {g.dtype}, {g.numel()} elements on "
                                       f"{g.device}; expected {c.dtype}, {self._numels[i]}, {self.device}")
                if not g.is_contiguous():
                    g = g.contiguous()
                ptrs[k] = g.data_ptr()
            grads.append(g)
        return grads, ptrs

    def _cached_grads(self, k: int, c: _Class) -> tuple[list[torch.Tensor | None], np.ndarray]:
        """_owned_grads, reusing the pointers found by the previous call of this step (the
        gradient objects are checked by identity, which costs far less than re-reading them)."""
        cached = self._grad_cache.get(k)
        if cached is not None:
            orig, grads, ptrs = cached
            if all(self.params[i].grad is g for i, g in zip(c.owned, orig)):
                return grads, ptrs
        grads, ptrs = self._owned_grads(c)
        self._grad_cache[k] = ([self.params[i].grad for i in c.owned], grads, ptrs)
        return grads, ptrs

    def _upload_table(self, c: _Class, grad_ptrs: np.ndarray, advance: bool) -> None:
        """Uploads class c's tensor table: the gradient pointers and, with ``advance``, the
        scalars of the next update (each tensor with a gradient at its step count + 1,
        optimizer.py:181); the counts themselves advance only when step() runs."""
        self._table_epoch += 1
        tab = c.table.np[:len(c.owned)]
        tab["grad"] = grad_ptrs
        if c.code != HA_F32 and self.world == 1:
            tab["param"] = np.fromiter((self.params[i].data.data_ptr() for i in c.owned), dtype=np.uint64,
                                       count=len(c.owned))
        if advance:
            idx = np.asarray(c.owned, dtype=np.int64)
            steps = np.ascontiguousarray(self._steps[idx] + (grad_ptrs != 0))
            _lib.call("ha_fill_step_scalars", len(c.owned), _lib.np_ptr(c.lrs), _lib.np_ptr(steps),
                      self.betas[0], self.betas[1], self.weight_decay, _lib.np_ptr(tab))
        c.table.upload()

    def _stage_step(self) -> None:
        """Uploads the next update's tables ahead of the norm's host read (which leaves the GPU
        idle until the host launches the update): step() then only launches, if nothing it
        depends on changed in between (the gradients, the tables, the step counts)."""
        staged = []
        for k, c in enumerate(self._classes):
            grads, ptrs = self._cached_grads(k, c)
            self._upload_table(c, ptrs, advance=True)
            staged.append((grads, ptrs))
        self._staged = (self._table_epoch, self.param_steps.version,
                        [self.params[i].grad for c in self._classes for i in c.owned], staged,
                        self._owned_param_ptrs())

    def _owned_param_ptrs(self) -> list[int]:
        """Addresses of the owned parameters (world 1: the tables point at them directly)."""
        return [self.params[i].data_ptr() for c in self._classes for i in c.owned] if self.world == 1 else []

    # ---------------------------------------------------------------- gradient landing
    def _setup_landing(self) -> None:
        """Gradient landing (p2p mode): a post-accumulate-grad hook on every parameter
        (the point where the reference's trainer hands the gradient over, train.py:268)
        pushes the pieces of the new gradient that belong to exchange rounds 0 and 1 to their
        owners' receive windows while backward is still running, on a separate stream, in
        buckets of HYBRIDAGENT_B200_LAND_BUCKET_BYTES (default 256 MiB) and at the end of each
        backward pass.  ``all_reduce_grads`` then pushes only the rest.  A gradient that lands
        again (a later backward of the same step) is pushed again; the last push wins.

        The pushes go to the copy engines (``land_ctas`` 0, the default), which take no SM from
        backward's kernels; HYBRIDAGENT_B200_LAND_CTAS=N > 0 runs them as a kernel of N CTAs
        walking the chunk list instead (measured on B200 at W=2: the copy engines cost backward
        4.4 ms for 16.4 GB moved, a 64-CTA kernel 12.9 ms, 8-32 CTAs too slow to finish within
        backward).  The copy tables of the kernel pushes go through a pinned arena (host) and its
        device twin, appended per push and rewound once the exchange has consumed them."""
        self._land_stream = torch.cuda.Stream(device=self.device)
        self._entry_of = {}
        n_pieces = n_chunks = 0
        for ci, c in enumerate(self._classes):
            for k, i in enumerate(c.layout.indices):
                self._entry_of[i] = (ci, k)
            n_pieces += int(c.land_mask.sum())
            n_chunks += int(((c.pieces.count[c.land_mask] + HA_ADAMW_CHUNK - 1) // HA_ADAMW_CHUNK).sum())
        # room for two landings of every gradient in one step before the arena is rewound
        self._land_cap = (max(2 * n_pieces, 1), max(2 * n_chunks, 1))
        csz, hsz = _lib.COPY_DTYPE.itemsize, _lib.CHUNK_DTYPE.itemsize
        self._land_copies = (torch.empty(self._land_cap[0] * csz, dtype=torch.uint8, pin_memory=True),
                             torch.empty(self._land_cap[0] * csz, dtype=torch.uint8, device=self.device))
        self._land_chunks = (torch.empty(self._land_cap[1] * hsz, dtype=torch.uint8, pin_memory=True),
                             torch.empty(self._land_cap[1] * hsz, dtype=torch.uint8, device=self.device))
        self._land_cursor = [0, 0]
        self._land_pending: list = []  # (class, entry, gradient, stream it was accumulated on)
        self._land_pending_bytes = 0
        self._land_bucket = int(os.environ.get("HYBRIDAGENT_B200_LAND_BUCKET_BYTES", str(256 << 20)))
        # 0: early pushes on the copy engines (no SM taken from backward); N > 0: a pushing
        # kernel on N CTAs (remote stores move ~6 GB/s per CTA, so it must take many SMs)
        self.land_ctas = int(os.environ.get("HYBRIDAGENT_B200_LAND_CTAS", "0"))
        self._land_ok = True         # no exchange of this optimizer is between its pushes and its update
        self._land_waited = False    # the landing stream already waits for the last update's barrier
        self._window_free = None     # event after that barrier
        self._land_callback = False  # an end-of-backward flush is queued
        me = weakref.ref(self)

        def hook(i):
            def on_landed(p):
                opt = me()
                if opt is not None:
                    opt._on_landed(i, p)
            return on_landed

        self._land_hooks = [p.register_post_accumulate_grad_hook(hook(i)) for i, p in enumerate(self.params)]
        self.landing_enabled = True
        # peers' host-side heartbeats, checked before every early push (which runs before any
        # deadline-bound collective): with a stale peer the push is left to all_reduce_grads
        self._liveness = None
        self.land_skipped = 0
        try:
            import torch.distributed as dist
            store = dist.distributed_c10d._get_default_store() if dist.is_initialized() else None
        except Exception:  # noqa: BLE001 -- no process-group store: no heartbeat
            store = None
        if store is not None:
            from .liveness import Heartbeat
            self._liveness = Heartbeat(store, self.rank, self.world,
                                       deadline_s=float(os.environ.get("HYBRIDAGENT_B200_LAND_DEADLINE_S", "3.0")))

    def _on_landed(self, i: int, p: torch.Tensor) -> None:
        """Post-accumulate-grad hook of parameter i (runs on the autograd engine's thread)."""
        if not (self.landing_enabled and self._land_ok):
            # the gradient changed (in place, keeping its identity) after any earlier early push:
            # forget that push so the exchange sends the gradient whole
            self._landed.pop(i, None)
            return
        ci, k = self._entry_of[i]
        c = self._classes[ci]
        g = p.grad
        if (g is None or g.dtype != c.dtype or g.device != self.device or g.numel() != self._numels[i]
                or not g.is_contiguous() or not len(c.land_pieces[k])):
            self._landed.pop(i, None)  # all_reduce_grads pushes it
            return
        self._landed[i] = (g, g._version)
        self._land_pending.append((ci, k, g, torch.cuda.current_stream(self.device)))
        self._land_pending_bytes += g.numel() * g.element_size()
        if not self._land_callback:
            self._land_callback = True
            torch.autograd.Variable._execution_engine.queue_callback(self._land_end_of_backward)
        if self._land_pending_bytes >= self._land_bucket:
            self._land_flush()

    def _land_end_of_backward(self) -> None:
        self._land_callback = False
        self._land_flush()

    def _land_flush(self) -> None:
        """Pushes the pending landed gradients' early pieces on the landing stream."""
        pending, self._land_pending, self._land_pending_bytes = self._land_pending, [], 0
        if not pending:
            return
        if self._liveness is not None and not self._liveness.all_fresh():
            # a peer's heartbeat is stale: push nothing into its memory now; the exchange sends
            # these gradients after its collective has confirmed every rank (or raised CommFailure)
            for ci, k, _, _ in pending:
                self._landed.pop(self._classes[ci].layout.indices[k], None)
            self.land_skipped += 1
            return
        land = self._land_stream
        with torch.cuda.device(self.device):
            for st in {st.cuda_stream: st for *_, st in pending}.values():
                land.wait_stream(st)  # the gradients are complete
            if not self._land_waited:
                if self._window_free is not None:
                    land.wait_event(self._window_free)  # every owner has read the previous exchange
                self._land_waited = True
            by_class: dict[int, list] = {}
            for ci, k, g, _ in pending:
                by_class.setdefault(ci, []).append((k, g))
            csz, hsz = _lib.COPY_DTYPE.itemsize, _lib.CHUNK_DTYPE.itemsize
            for ci, items in by_class.items():
                c = self._classes[ci]
                idx = np.concatenate([c.land_pieces[k] for k, _ in items])
                base = np.concatenate([np.full(len(c.land_pieces[k]), g.data_ptr(), dtype=np.uint64)
                                       for k, g in items])
                copies, chunks = layout.landing_batch(base + c.piece_src_bytes[idx], c.piece_dst[idx],
                                                      c.pieces.count[idx], HA_ADAMW_CHUNK)
                if self.land_ctas == 0:  # copy engines: the host table is read by the calls themselves
                    _lib.call("ha_copy_async", _lib.np_ptr(copies), len(copies), c.packed_param.element_size(),
                              land.cuda_stream)
                    self.land_launches += 1
                    continue
                a, b = self._land_cursor
                if a + len(copies) > self._land_cap[0] or b + len(chunks) > self._land_cap[1]:
                    land.synchronize()  # every earlier upload has been consumed: rewind the arena
                    a = b = 0
                hc, dc = self._land_copies
                hk, dk = self._land_chunks
                hc.numpy()[a * csz:(a + len(copies)) * csz] = copies.view(np.uint8)
                hk.numpy()[b * hsz:(b + len(chunks)) * hsz] = chunks.view(np.uint8)
                with torch.cuda.stream(land):
                    dc[a * csz:(a + len(copies)) * csz].copy_(hc[a * csz:(a + len(copies)) * csz], non_blocking=True)
                    dk[b * hsz:(b + len(chunks)) * hsz].copy_(hk[b * hsz:(b + len(chunks)) * hsz], non_blocking=True)
                _lib.call("ha_gather_capped", dc.data_ptr() + a * csz, dk.data_ptr() + b * hsz, len(chunks),
                          HA_ADAMW_CHUNK, c.packed_param.element_size(), self.land_ctas, land.cuda_stream)
                self.launches += 1
                self.land_launches += 1
                self._land_cursor = [a + len(copies), b + len(chunks)]
            for _, _, g, _ in pending:
                g.record_stream(land)  # the allocator keeps it until the push has read it

    def _land_join(self) -> None:
        """Start of an exchange: flushes what is pending and orders the current stream after
        every early push (the arena is rewound once the next host read has waited for it)."""
        self._land_flush()
        self._land_callback = False
        torch.cuda.current_stream(self.device).wait_stream(self._land_stream)

    # ---------------------------------------------------------------- gradient landing, world size 1
    def _setup_landing_local(self) -> None:
        """Gradient landing at world size 1: the norm's square sums are taken while backward is
        still running.  A post-accumulate-grad hook on every parameter (train.py:268's
        ``loss.backward()`` hands each gradient over there) queues the gradient; every
        HYBRIDAGENT_B200_LAND_BUCKET_BYTES and at the end of each backward pass the queued
        gradients' sums of squares are launched on a side stream (one ``ha_grad_sumsq_ctas`` per
        dtype class, each into its own fp64 slot, on at most ``land_ctas`` CTAs -- 0: one per
        chunk -- so that backward keeps the other SMs).  ``clip_grad_norm`` then adds the slots instead of
        reading every gradient again -- if every owned gradient landed exactly once and is the
        same object, unmodified (torch's version counter), that it is now; otherwise it takes the
        full pass.  Results are the same sums of the same squares, grouped per landing."""
        self._lland = True
        self._lland_stream = torch.cuda.Stream(device=self.device)
        self._lland_bucket = int(os.environ.get("HYBRIDAGENT_B200_LAND_BUCKET_BYTES", str(256 << 20)))
        self.land_ctas = int(os.environ.get("HYBRIDAGENT_B200_LAND_CTAS", "0"))
        n_chunks = sum(c.sumsq_chunks[1] for c in self._classes)
        self._lland_cap = (max(2 * len(self.params), 1), max(2 * n_chunks, 1))  # tensors, chunks (two landings each)
        csz, tsz = _lib.CHUNK_DTYPE.itemsize, _lib.TENSOR_DTYPE.itemsize
        dev = self.device
        self._lland_tab = (torch.empty(self._lland_cap[0] * tsz, dtype=torch.uint8, pin_memory=True),
                           torch.empty(self._lland_cap[0] * tsz, dtype=torch.uint8, device=dev))
        self._lland_chk = (torch.empty(self._lland_cap[1] * csz, dtype=torch.uint8, pin_memory=True),
                           torch.empty(self._lland_cap[1] * csz, dtype=torch.uint8, device=dev))
        self._lland_partials = torch.empty(self._lland_cap[1], dtype=torch.float64, device=dev)
        self._lland_out = torch.zeros(self._lland_cap[0], dtype=torch.float64, device=dev)
        self._lland_out_host = torch.zeros(self._lland_cap[0], dtype=torch.float64, pin_memory=True)
        self._lland_class_of = {i: ci for ci, c in enumerate(self._classes) for i in c.owned}
        self._lland_reset()
        me = weakref.ref(self)

        def hook(i):
            def on_landed(p):
                opt = me()
                if opt is not None and opt.landing_enabled:
                    opt._lland_on_landed(i, p)
            return on_landed

        self._land_hooks = [p.register_post_accumulate_grad_hook(hook(i)) for i, p in enumerate(self.params)]
        self.landing_enabled = True

    def _lland_reset(self) -> None:
        self._lland_pending: list = []  # (parameter index, gradient, stream it was accumulated on)
        self._lland_bytes = 0
        self._lland_seen: dict[int, tuple] = {}  # parameter index -> (gradient, its version when summed)
        self._lland_slots = 0     # fp64 slots written so far this step
        self._lland_cursor = [0, 0]  # table entries, chunks used in the arenas
        self._lland_valid = True  # no gradient summed twice, nothing out of room, no in-place clip
        self._lland_callback = False

    def _lland_on_landed(self, i: int, p: torch.Tensor) -> None:
        g = p.grad
        if g is None or i not in self._lland_class_of or not g.is_contiguous():
            self._lland_valid = False
            return
        self._lland_pending.append((i, g, torch.cuda.current_stream(self.device)))
        self._lland_bytes += g.numel() * g.element_size()
        if not self._lland_callback:
            self._lland_callback = True
            torch.autograd.Variable._execution_engine.queue_callback(self._lland_end_of_backward)
        if self._lland_bytes >= self._lland_bucket:
            self._lland_flush()

    def _lland_end_of_backward(self) -> None:
        self._lland_callback = False
        self._lland_flush()

    def _lland_flush(self) -> None:
        """Launches the sums of squares of the queued gradients on the landing stream."""
        pending, self._lland_pending, self._lland_bytes = self._lland_pending, [], 0
        if not pending:
            return
        land = self._lland_stream
        csz, tsz = _lib.CHUNK_DTYPE.itemsize, _lib.TENSOR_DTYPE.itemsize
        with torch.cuda.device(self.device):
            for st in {st.cuda_stream: st for *_, st in pending}.values():
                land.wait_stream(st)  # the gradients are complete
            by_class: dict[int, list] = {}
            for i, g, _ in pending:
                if i in self._lland_seen:
                    self._lland_valid = False  # landed again: its earlier sum is stale
                by_class.setdefault(self._lland_class_of[i], []).append((i, g))
            for ci, items in by_class.items():
                c = self._classes[ci]
                numels = [g.numel() for _, g in items]
                chunks = layout.chunk_table(numels, HA_SUMSQ_CHUNK)
                t0, k0 = self._lland_cursor
                if (t0 + len(items) > self._lland_cap[0] or k0 + len(chunks) > self._lland_cap[1]
                        or self._lland_slots >= self._lland_cap[0]):
                    self._lland_valid = False  # out of room: clip_grad_norm takes the full pass
                    continue
                tab = np.zeros(len(items), dtype=_lib.TENSOR_DTYPE)
                tab["grad"] = [g.data_ptr() for _, g in items]
                tab["numel"] = numels
                ht, dt = self._lland_tab
                hk, dk = self._lland_chk
                ht.numpy()[t0 * tsz:(t0 + len(items)) * tsz] = tab.view(np.uint8)
                hk.numpy()[k0 * csz:(k0 + len(chunks)) * csz] = chunks.view(np.uint8)
                with torch.cuda.stream(land):
                    dt[t0 * tsz:(t0 + len(items)) * tsz].copy_(ht[t0 * tsz:(t0 + len(items)) * tsz], non_blocking=True)
                    dk[k0 * csz:(k0 + len(chunks)) * csz].copy_(hk[k0 * csz:(k0 + len(chunks)) * csz], non_blocking=True)
                slot = self._lland_slots
                _lib.call("ha_grad_sumsq_ctas", dt.data_ptr() + t0 * tsz, dk.data_ptr() + k0 * csz, len(chunks),
                          HA_SUMSQ_CHUNK, c.code, self._lland_partials.data_ptr() + k0 * 8,
                          self._lland_out.data_ptr() + slot * 8, self.land_ctas, land.cuda_stream)
                self.launches += 2 if len(chunks) else 1
                self._lland_slots += 1
                self._lland_cursor = [t0 + len(items), k0 + len(chunks)]
                for i, g in items:
                    self._lland_seen[i] = (g, g._version)
            for _, g, _ in pending:
                g.record_stream(land)  # the allocator keeps it until its sum has read it

    def _lland_ready(self) -> bool:
        """Every owned gradient present now landed once, unchanged since; none landed that is
        gone."""
        if not (self._lland and self._lland_valid and self._lland_slots):
            return False
        present = 0
        for c in self._classes:
            for i in c.owned:
                g = self.params[i].grad
                if g is None:
                    continue
                present += 1
                seen = self._lland_seen.get(i)
                if seen is None or seen[0] is not g or seen[1] != g._version:
                    return False
        return present == len(self._lland_seen)

    # ---------------------------------------------------------------- reference surface
    def zero_grad(self, set_to_none: bool = True) -> None:
        """optimizer.py:88-93."""
        self._pending_clip = None
        self._fused_sumsq = None
        self._grad_cache = {}
        self._staged = None
        self._landed = {}  # what was pushed early no longer matches the gradients
        if self._lland:
            self._lland_stream.synchronize()  # the arenas are rewritten by the next landings
            self._lland_reset()
        elif self._land_hooks:  # (a backward that raised may have left both behind)
            self._land_pending, self._land_pending_bytes = [], 0
            self._land_callback = False
        for parameter in self.params:
            if set_to_none:
                parameter.grad = None
            elif parameter.grad is not None:
                parameter.grad.zero_()

    @_nvtx
    @torch.no_grad()
    def all_reduce_grads(self) -> None:
        """Sum every rank's gradient onto its owner (optimizer.py:95-143).  Tensors with no
        gradient on any rank keep grad=None; owners receive views of the reduced segment
        and every other rank None.  All ranks must call it."""
        if self.world == 1:
            return
        self.apply_pending_clip()
        with torch.cuda.device(self.device):
            # everything that reads the parameters' Python attributes happens before the mask is
            # synchronised, overlapping the GPU's earlier work (it dominates with ~10^4 tensors)
            keep = []  # gradients that must stay alive until the move kernel has read them
            p2p = self.comm_mode == "p2p"
            landed = self._landed
            if self._land_hooks:
                self._land_join()
            local = self._used_local.numpy()
            local[:] = 0
            class_ptrs = []
            for c in self._classes:
                ptrs = np.zeros(len(c.layout.indices), dtype=np.uint64)
                esz = c.packed_param.element_size()
                base = c.packed_param.data_ptr()
                for k, i in enumerate(c.layout.indices):
                    p = self.params[i]
                    if p.data.data_ptr() != base + (self.owner[i] * c.layout.seg_len + c.layout.offset[i]) * esz:
                        raise RuntimeError(f"parameter {i} was re-bound after the optimizer was built")
                    g = p.grad
                    if g is None:
                        continue
                    local[i] = 1
                    if g.dtype != c.dtype or g.numel() != self._numels[i] or g.device != self.device:
                        raise RuntimeError(f"gradient of tensor {i}: {g.dtype} x {g.numel()} on {g.device}")
                    if not g.is_contiguous():
                        g = g.contiguous()
                    keep.append(g)
                    ptrs[k] = g.data_ptr()
                class_ptrs.append(ptrs)
            # the copy tables depend only on this rank's gradients (a tensor no rank uses has no
            # gradient here either: zero-filled, optimizer.py:111-114), so they are built and
            # uploaded before the mask's all-reduce and the host waits only for that
            for ci, (c, ptrs) in enumerate(zip(self._classes, class_ptrs)):
                if p2p:  # each piece reads its part of its tensor's gradient (0: zero-fill; gaps: zeros)
                    done = None
                    if landed:  # pieces pushed while their gradient landed, gradient unchanged: skipped
                        done = np.zeros(len(c.layout.indices), dtype=bool)
                        for i, (g, version) in landed.items():
                            # the same object, not modified in place since its push (in-place ops
                            # such as p.grad.div_() bump the version counter)
                            if self._entry_of[i][0] == ci and self.params[i].grad is g and g._version == version:
                                done[self._entry_of[i][1]] = True
                    src = layout.piece_sources(c.pieces, ptrs, c.packed_param.element_size(), c.piece_dst, done)
                    c.move.np["src"][:len(src)] = src
                else:  # equal to dst when the gradient already lives in its slot
                    c.move.np["src"][:len(ptrs)] = ptrs
                c.move.upload()
            T = len(self.params)
            local[T:] = self._detect_dirty()  # every rank learns every rank's dirty tensors
            self._used_dev.copy_(self._used_local, non_blocking=True)  # no host wait: a peer may be missing
            self._comm.all_reduce_max(self._used_dev, HA_U8)
            # a rank that stopped answering ends here (CommFailure), before any peer store
            both = self._comm.read(self._used_dev, self._used_host, "all-reduce(max) of the used mask")
            both = both.numpy().astype(bool)
            used = both[:T]
            self._dirty |= both[T:]
            self._last_used = used
            if self._land_hooks:  # the early pushes have all completed: rewind their arena
                self._land_cursor = [0, 0]
                self._land_waited = False
                self._land_ok = False  # until the update's barrier frees the windows again
                self._landed = {}
            if p2p:
                self._exchange_rounds()
            else:
                self._phase("pack", True)
                for c in self._classes:
                    if c.move_chunks[1]:
                        _lib.call("ha_gather", c.move.ptr, c.move_chunks[0].data_ptr(), c.move_chunks[1],
                                  HA_ADAMW_CHUNK, c.grad_buf.element_size(), self._stream())
                        self.launches += 1
                self._phase("pack", False)
                self._phase("reduce_scatter", True)
                for c in self._classes:
                    own = c.grad_buf.data_ptr() + self.rank * c.layout.seg_len * c.grad_buf.element_size()
                    self._comm.reduce_scatter(c.grad_buf.data_ptr(), own, c.layout.seg_len, c.code)
                self._phase("reduce_scatter", False)
            del keep
            self._grad_cache = {}
            for c in self._classes:
                for i in c.layout.indices:
                    if used[i] and self.owner[i] == self.rank:
                        self.params[i].grad = c.grad_view[i]
                    else:
                        self.params[i].grad = None
            # the square sums of exactly these gradients are ready (p2p): clip_grad_norm reuses
            # them unless an owned gradient is replaced before it runs
            self._fused_sumsq = [self.params[i].grad for c in self._classes for i in c.owned] if p2p else None

    @_nvtx
    @torch.no_grad()
    def clip_grad_norm(self, max_norm: float) -> float:
        """Global L2 norm of the owned gradients (all ranks), clipping to max_norm
        (optimizer.py:145-160).  Returns the pre-clip norm."""
        self.apply_pending_clip()
        with torch.cuda.device(self.device):
            fused = self._fused_sumsq
            self._fused_sumsq = None
            reuse = fused is not None and all(
                self.params[i].grad is g for g, i in zip(fused, (i for c in self._classes for i in c.owned)))
            landed = False
            if self._lland:  # world 1: the square sums taken while the gradients landed
                self._lland_flush()
                self._lland_callback = False
                landed = self._lland_ready()
            if landed:
                torch.cuda.current_stream().wait_stream(self._lland_stream)
                n_slots = self._lland_slots
                partial = self._read_local(self._lland_out[:n_slots], self._lland_out_host[:n_slots])
                self.land_norm_steps += 1
            else:
                # (the contiguous copies of strided gradients must outlive the launches)
                keep = None if reuse else self._launch_sumsq()  # noqa: F841
                if self.world > 1 and reuse:  # the exchange's square sums, one per class and round
                    self._comm.all_reduce_sum(self._norm_rounds, HA_F64)
                    self._stage_step()
                    partial = self._comm.read(self._norm_rounds, self._norm_rounds_host,
                                              "all-reduce(sum) of the norm").reshape(-1).tolist()
                elif self.world > 1:
                    self._comm.all_reduce_sum(self._norm_buf, HA_F64)
                    self._stage_step()
                    partial = self._comm.read(self._norm_buf, self._norm_host,
                                              "all-reduce(sum) of the norm").tolist()
                else:
                    partial = self._read_local(self._norm_buf, self._norm_host)
        total = np.float32(sum(partial))  # the reference's total is an fp32 tensor
        norm = float(np.sqrt(total))      # float(total.sqrt()), optimizer.py:154
        if max_norm > 0 and norm > max_norm:
            self._pending_clip = float(max_norm) / (norm + 1e-6)  # optimizer.py:156
        return norm

    def _launch_sumsq(self) -> list:
        """One ``ha_grad_sumsq`` per dtype class over its owned gradients into ``_norm_buf``;
        returns the gradient lists, whose contiguous copies must outlive the launches."""
        keep = []
        for k, c in enumerate(self._classes):
            grads, ptrs = self._cached_grads(k, c)
            keep.append(grads)
            self._upload_table(c, ptrs, advance=False)
        self._phase("sumsq", True)
        for k, c in enumerate(self._classes):
            chunks, n = c.sumsq_chunks
            _lib.call("ha_grad_sumsq", c.table.ptr, None if chunks is None else chunks.data_ptr(), n,
                      HA_SUMSQ_CHUNK, c.code, c.partials.data_ptr(), self._norm_buf[k:].data_ptr(), self._stream())
            self.launches += 2 if n else 1
        self._phase("sumsq", False)
        return keep

    def _read_local(self, dev: torch.Tensor, host: torch.Tensor) -> list:
        """World size 1: copies the fp64 sums to pinned host memory, stages the next step's
        tables while the copy is in flight, and returns the sums."""
        host.copy_(dev, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        self._stage_step()
        ev.synchronize()
        return host.tolist()

    @_nvtx
    @torch.no_grad()
    def apply_pending_clip(self) -> None:
        """Scales the owned gradients in place by the factor the last clip_grad_norm chose
        (the reference's ``grad.mul_(scale)``, optimizer.py:157-159); no-op if none."""
        if self._pending_clip is None:
            return
        scale, self._pending_clip = self._pending_clip, None
        self._fused_sumsq = None  # the gradients change below
        if self._lland:
            self._lland_valid = False  # (in place, by this library's kernel: torch sees no new version)
        self._grad_cache = {}
        with torch.cuda.device(self.device):
            keep = []
            for c in self._classes:
                grads, ptrs = self._owned_grads(c)
                keep.append(grads)
                self._upload_table(c, ptrs, advance=False)
                sc = _lib.AdamwScalars()
                _lib.call("ha_make_scalars", self.betas[0], self.betas[1], self.eps, self.weight_decay, c.code, 1,
                          scale, ctypes.byref(sc))
                chunks, n = c.adamw_chunks
                if n:
                    _lib.call("ha_scale_grads", c.table.ptr, chunks.data_ptr(), n, HA_ADAMW_CHUNK, c.code,
                              sc.clip_mult, self._stream())
                    self.launches += 1
                for i, g in zip(c.owned, grads):  # strided gradients were scaled in a contiguous copy
                    if g is not None and g is not self.params[i].grad:
                        self.params[i].grad.copy_(g)

    @_nvtx
    @torch.no_grad()
    def step(self) -> None:
        """Fused AdamW over the owned tensors with a gradient, then the parameter
        all-gather (optimizer.py:162-194)."""
        self.step_count += 1
        scale, self._pending_clip = self._pending_clip, None
        with torch.cuda.device(self.device):
            launches, keep = [], []
            updated = np.zeros(len(self.params), dtype=bool)  # tensors this step writes (the used set)
            staged, self._staged = self._staged, None
            if staged is not None and (staged[0] != self._table_epoch or staged[1] != self.param_steps.version or
                                       any(self.params[i].grad is not g for g, i in
                                           zip(staged[2], (i for c in self._classes for i in c.owned)))):
                staged = None  # something changed since clip_grad_norm staged the tables
            if staged is not None and staged[4] != self._owned_param_ptrs():
                staged = None  # a parameter was re-bound: its table entry must be rewritten
            for k, c in enumerate(self._classes):
                if staged is not None:
                    grads, ptrs = staged[3][k]
                else:
                    grads, ptrs = self._cached_grads(k, c)
                    self._upload_table(c, ptrs, advance=True)
                keep.append(grads)
                idx = np.asarray(c.owned, dtype=np.int64)
                self._steps[idx[ptrs != 0]] += 1  # optimizer.py:181, only tensors that have a gradient
                updated[idx[ptrs != 0]] = True
                sc = _lib.AdamwScalars()
                _lib.call("ha_make_scalars", self.betas[0], self.betas[1], self.eps, self.weight_decay, c.code,
                          0 if scale is None else 1, 0.0 if scale is None else scale, ctypes.byref(sc))
                launches.append((c, sc))
            if self.world == 1:
                self._dirty |= self._detect_dirty()
            elif self._last_used is not None:
                updated = self._last_used  # every rank's owners update exactly the used tensors
            else:  # no all_reduce_grads before this step: clear nothing (the set must stay collective)
                updated = np.zeros(len(self.params), dtype=bool)
            self._last_used = None
            p2p = self.comm_mode == "p2p"
            # changed-groups-only writes (16-bit classes) unless some parameter or master was written
            # behind the optimizer's back: then this step writes everything, as the reference does
            dense = not self.delta_writes or bool(self._dirty.any())
            self._dense_this_step = dense
            self.dense_steps += dense
            self._phase("adamw", True)
            ce_gather = p2p and self.gather_mode == "ce"
            main = torch.cuda.current_stream()
            for c, sc in launches:
                chunks, n = c.adamw_chunks
                if c.changed_event is not None and c.changed_event.query():  # the last count has landed
                    c.last_changed = int(c.changed_host[0])
                    c.delta_next = c.last_changed <= self.delta_max_fraction * max(c.groups, 1)
                    c.changed_event = None
                elif not c.delta_next:
                    c.full_run += 1
                    if c.full_run >= 8:  # look again: the learning rate or the gradients may have changed
                        c.delta_next, c.full_run = True, 0
                if (n and not dense and c.delta_next and c.code != HA_F32 and not ce_gather
                        and self.comm_mode != "nccl"):
                    _lib.call("ha_memset", c.changed_dev.data_ptr(), 0, 8, self._stream())
                    _lib.call("ha_adamw_step_delta", c.table.ptr, chunks.data_ptr(), n, HA_ADAMW_CHUNK, c.code,
                              ctypes.byref(sc), ctypes.byref(c.peers) if p2p else None, c.changed_dev.data_ptr(),
                              self._stream())
                    self.launches += 1
                    c.changed_host.copy_(c.changed_dev, non_blocking=True)
                    c.changed_event = torch.cuda.Event()
                    c.changed_event.record()
                elif n and ce_gather:  # update in parts; the copy engines send each finished part to the peers
                    esz = c.packed_param.element_size()
                    for (c0, nc, _, _), copies in zip(c.gather_parts, c.gather_copies):
                        _lib.call("ha_adamw_step", c.table.ptr, chunks.data_ptr() + c0 * _lib.CHUNK_DTYPE.itemsize,
                                  nc, HA_ADAMW_CHUNK, c.code, c.code, ctypes.byref(sc), main.cuda_stream)
                        self.launches += 1
                        done = torch.cuda.Event()
                        done.record(main)
                        for st, cp in zip(self._gather_streams, copies):
                            st.wait_event(done)
                            _lib.call("ha_copy_async", _lib.np_ptr(cp), 1, esz, st.cuda_stream)
                elif n and p2p:  # the update also writes each new parameter into every peer's copy
                    _lib.call("ha_adamw_step_peers", c.table.ptr, chunks.data_ptr(), n, HA_ADAMW_CHUNK, c.code,
                              c.code, ctypes.byref(sc), ctypes.byref(c.peers), self._stream())
                    self.launches += 1
                elif n:
                    _lib.call("ha_adamw_step", c.table.ptr, chunks.data_ptr(), n, HA_ADAMW_CHUNK, c.code, c.code,
                              ctypes.byref(sc), self._stream())
                    self.launches += 1
            for st in self._gather_streams:
                main.wait_stream(st)
            self._phase("adamw", False)
            # a dirty tensor without a gradient is not updated, but the reference still broadcasts
            # every parameter from its owner (optimizer.py:192-194): do the same with one all-gather
            regather = self.world > 1 and bool((self._dirty & ~updated).any())
            if p2p:
                self._phase("barrier", True)
                self._barrier()  # peers use their parameters only after every rank's stores landed
                self._phase("barrier", False)
                if regather:
                    self._all_gather_params()
                if self._land_hooks:  # every owner has read its windows: early pushes may start
                    self._window_free = torch.cuda.Event()
                    self._window_free.record()
                    self._land_ok = True
            elif self.world > 1:
                self._all_gather_params()
            # written in full (dense) or by changed groups from a clean state: clean now, on every rank
            self._dirty &= ~updated

    def write_stats(self) -> dict:
        """How the parameter copies were written by the latest update: ``mode`` ("changed groups"
        or "full"), ``changed_groups`` (4-element groups stored by the latest changed-groups
        update, all classes; waits for its count) and ``groups`` (4-element groups owned)."""
        for c in self._classes:
            if c.changed_event is not None:
                c.changed_event.synchronize()
                c.last_changed = int(c.changed_host[0])
                c.delta_next = c.last_changed <= self.delta_max_fraction * max(c.groups, 1)
                c.changed_event = None
        bf = [c for c in self._classes if c.code != HA_F32]
        delta = bool(bf) and not self._dense_this_step and all(c.last_changed is not None for c in bf)
        return {"mode": "changed groups" if delta else "full", "changed_groups": self.last_changed_groups,
                "groups": sum(c.groups for c in bf)}

    @property
    def last_changed_groups(self) -> int | None:
        """4-element parameter groups stored by the most recent changed-groups update whose
        count has been read back (all classes), or None before the first."""
        counts = [c.last_changed for c in self._classes if c.last_changed is not None]
        return sum(counts) if counts else None

    def _all_gather_params(self) -> None:
        """Every rank's packed parameter segments from their owners (NCCL, in place)."""
        self._phase("all_gather", True)
        for c in self._classes:
            own = c.packed_param.data_ptr() + self.rank * c.layout.seg_len * c.packed_param.element_size()
            self._comm.all_gather(own, c.packed_param.data_ptr(), c.layout.seg_len, c.code)
        self._phase("all_gather", False)

    def state_summary(self) -> str:
        """optimizer.py:196-199."""
        return (f"ZeRO-1 FP32 AdamW: {len(self.params)} tensors; rank {self.rank} owns "
                f"{self.owned_numel / 1e6:.1f}M parameters")

    # ---------------------------------------------------------------- checkpointing (new surface)
    def state_dict(self) -> dict:
        """This rank's shard: fp32 master / exp_avg / exp_avg_sq and the step counts of its
        owned tensors (CPU copies), keyed by flat parameter index, plus what identifies the
        layout.  Loading it into an optimizer built over the same parameters, rank and
        world size resumes bit-identically."""
        torch.cuda.current_stream(self.device).synchronize()
        owned = list(self.param_steps)
        return {
            "format": STATE_FORMAT,
            "world": self.world,
            "rank": self.rank,
            "step_count": self.step_count,
            "owner": list(self.owner),
            "numels": list(self._numels),
            "lrs": list(self.lrs),
            "betas": self.betas,
            "eps": self.eps,
            "weight_decay": self.weight_decay,
            "param_steps": {i: int(self._steps[i]) for i in owned},
            "master": {i: self.master[i].detach().to("cpu", copy=True) for i in owned},
            "exp_avg": {i: self.exp_avg[i].detach().to("cpu", copy=True) for i in owned},
            "exp_avg_sq": {i: self.exp_avg_sq[i].detach().to("cpu", copy=True) for i in owned},
        }

    @torch.no_grad()
    def load_state_dict(self, state: dict) -> None:
        if state.get("format") != STATE_FORMAT:
            raise ValueError(f"not a {STATE_FORMAT} state dict")
        for key, mine in (("world", self.world), ("rank", self.rank), ("owner", list(self.owner)),
                          ("numels", list(self._numels))):
            if state[key] != mine:
                raise ValueError(f"state dict {key} does not match this optimizer")
        owned = list(self.param_steps)
        if sorted(state["param_steps"]) != sorted(owned):
            raise ValueError("state dict holds a different set of owned tensors")
        for i in owned:
            for name, dst in (("master", self.master[i]), ("exp_avg", self.exp_avg[i]),
                              ("exp_avg_sq", self.exp_avg_sq[i])):
                src = state[name][i]
                if src.shape != dst.shape:
                    raise ValueError(f"{name}[{i}] has shape {tuple(src.shape)}, expected {tuple(dst.shape)}")
                dst.copy_(src.to(dst.device, torch.float32))
            self._steps[i] = int(state["param_steps"][i])
        self.step_count = int(state["step_count"])
        self._staged = None
        self._pending_clip = None
        torch.cuda.current_stream(self.device).synchronize()

    def close(self) -> None:
        """Releases the peer mappings and the NCCL communicator (world_size > 1).  Call it on
        every rank after the last step: it waits for all of this rank's work (pushes, sums,
        early pushes included) and, at world > 1, for every rank to reach it (a barrier under
        the communicator's deadline), so no rank releases memory a peer still writes."""
        self._release(collective=True)

    def _release(self, collective: bool) -> None:
        for h in getattr(self, "_land_hooks", []):
            h.remove()
        self._land_hooks = []
        if getattr(self, "_liveness", None) is not None:
            self._liveness.stop()
            self._liveness = None
        self.landing_enabled = False
        if getattr(self, "_peer_map", None) is not None:
            torch.cuda.synchronize(self.device)  # every stream of this rank, peer stores included
            if collective and self._comm is not None and self._comm.failure is None:
                with torch.cuda.device(self.device):
                    self._barrier()
                    self._comm.read(self._barrier_buf, torch.zeros(1, dtype=torch.int32, pin_memory=True),
                                    "barrier before releasing the peer mappings")
            self._peer_map.close()
            self._peer_map = None
        if getattr(self, "_comm", None) is not None:
            self._comm.close()
            self._comm = None

    def __del__(self):
        try:
            self._release(collective=False)  # never a collective from the garbage collector
        except Exception:
            pass

