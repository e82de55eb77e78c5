"""B200 HAL: the NumpyBackend surface on device arenas, streams and events.

Drop-in for ``backend.hal_numpy.NumpyBackend`` (backend/hal_numpy.py:12-189)
with the same method names, argument meanings and error behaviour:

* ``CudaBackendConfig(num_dpus, mram_bytes_per_dpu, allow_device_to_device=False)``;
  each simulated DPU is one GPU rank with a zero-initialised device arena of
  ``mram_bytes_per_dpu`` bytes (the planner's three zones live inside it);
* ``copy_to_dpu / copy_from_dpu / write_local / read_local / push_xfer`` move
  bytes between host arrays and an arena, with the reference's bounds check
  (``ValueError("invalid MRAM range ...")``);
* ``submit(cmd) -> Event``, ``wait(event, timeout)``, ``query(event)``: each rank
  is one CUDA stream, so same-rank commands are ordered; ``waits`` become
  ``cudaStreamWaitEvent`` between streams; duplicate / unknown ids raise at
  submit, every other failure surfaces at ``wait``; ``dma_in`` snapshots its host
  payload at submit; device-to-device copies are refused at construction.

Differences that follow from real hardware:

* ``register_kernel`` functions are called synchronously at submit and must only
  enqueue device work on ``hal.stream(dpu_id)`` (a CUDA launch never blocks the
  caller);
* ``register_plan`` compiles every command of a plan once: launches become
  prebuilt C-ABI calls, host nodes run on device against a device-resident copy
  of the host location, and each redistribute edge (its collect transfers, host
  combine and writebacks) becomes one device collective executed at the combine
  command -- the ordered rank-sequence sum for Partial -> Replicate (bit-exact
  with comm/lowering.py:137-150) or one batched copy for all_gather /
  all_to_all / scatter.  No step of a plan touches the CPU;
* two process layouts: one process driving every rank (ranks mapped
  round-robin onto the visible GPUs, peers read over NVLink), or one process
  per GPU under ``torch.distributed`` (``rank`` set), where each process runs its
  own rank's commands plus the host commands, and combines are NCCL
  collectives.

``capture(plan)`` records one execution of a static plan into a CUDA graph
(the plan's inputs are device buffers, so a replay is a full step).
"""

from __future__ import annotations

import time
from dataclasses import dataclass, field

import numpy as np

from backend import _native as nat
from backend.cuda_kernels import lower_host_op, lower_launch
from contracts.exec_plan import Access

try:
    import torch
except ImportError as exc:  # pragma: no cover - torch is the device-memory plumbing
    raise ImportError("backend.hal_cuda needs PyTorch for device memory and streams") from exc


def _np_dtype(name) -> np.dtype:
    if isinstance(name, np.dtype):
        return name
    if str(name) == "bfloat16":
        import ml_dtypes

        return np.dtype(ml_dtypes.bfloat16)
    return np.dtype(name)


@dataclass
class CudaBackendConfig:
    num_dpus: int
    mram_bytes_per_dpu: int
    allow_device_to_device: bool = False
    devices: tuple[int, ...] | None = None  # single process: GPUs the ranks are spread over
    rank: int | None = None  # one process per GPU: this process's rank (torch.distributed)
    # One process per GPU, Partial->Replicate edges:
    #   "ordered" (default) NCCL all_gather of the partials + the rank-order sum kernel;
    #   "p2p"     small edges as one kernel over NVLink peer memory (backend/p2p.py) with
    #             the low-latency protocol (epoch-tagged 64-bit words, no fences), large
    #             ones as "ordered";
    #   "fused"   as "p2p", and linear -> all_reduce -> add chains as one kernel;
    #   "nccl"    NCCL all_reduce (not bit-exact).
    # All but "nccl" give the bit-exact rank-order sum of comm/lowering.py.
    allreduce: str = "ordered"
    # "ordered" edges of at least this many bytes (0: none) run as an all_to_all of column
    # slices, the rank-order sum of one slice per rank, and an all_gather of the sums:
    # 2(N-1)/N of the tensor per rank instead of the all_gather's (N-1), same bits.
    allreduce_split_bytes: int = 0
    # One process per GPU, "ordered" or "p2p": fold the residual `add` that consumes an
    # all_reduce into the combine's rank-order sum kernel (pim_ordered_sum_add, or the P2P
    # kernel's pim_allreduce_p2p_add; same bits, one launch and one pass over the sum fewer).
    combine_add: bool = False
    # Decode (rows <= 8): compute each layer's attention at the end of its attn_in launch
    # (the CTA that writes a head's last q / k / v value computes that head) instead of
    # launching the attention kernel.
    fuse_attention: bool = False
    # Decode with one activation row, at TP = 1 or (one process per GPU) with
    # allreduce="fused": run each layer's five commands (attn_in, attention, o_proj +
    # residual, mlp_in, down + residual; at TP > 1 with their all-reduces) as ONE launch
    # of the layer kernel (pim_decode_layer; grid-wide barriers between the phases, the
    # next phase's weights streaming across each barrier).
    decode_layer: bool = False
    # The whole decode step -- every layer and the final norm + lm_head -- as ONE launch
    # (pim_decode_step; a grid barrier between layers instead of a kernel boundary), under
    # the conditions of decode_layer (which it implies).
    decode_step: bool = False


_ITEM = {"float32": 4, "bfloat16": 2, "int32": 4}


def _on_rank(m, rank: int) -> bool:
    """Whether command ``m`` runs on ``rank``'s stream or on the host."""
    return m.dpu_id is None or int(m.dpu_id) == rank


def _window_clear(window, rank: int, touched, written, edge=None, host_writes: bool = False) -> bool:
    """No command of ``rank`` or of the host in ``window`` (the transfers of redistribute
    edge ``edge`` aside) reads or writes an interval of ``touched``, writes one of
    ``written`` or, with ``host_writes``, writes the host location."""
    for m in window:
        if not _on_rank(m, rank) or (edge is not None and m.payload.get("edge") == edge):
            continue
        if (any(a.overlaps(t) for a in list(m.reads) + list(m.writes) for t in touched)
                or any(a.overlaps(w) for a in m.writes for w in written)
                or (host_writes and any(a.loc == ("host", None) for a in m.writes))):
            return False
    return True


def _read_before_overwritten(after, rank: int, acc, skip=None, edge=None) -> bool:
    """Whether a command of ``rank`` or of the host in ``after`` (``skip`` and the transfers of
    ``edge`` aside) reads ``acc`` before one overwrites it."""
    for m in after:
        if not _on_rank(m, rank) or m is skip or (edge is not None and m.payload.get("edge") == edge):
            continue
        if any(a.overlaps(acc) for a in m.reads):
            return True
        if any(a.overlaps(acc) for a in m.writes):
            return False
    return False


def _noop() -> None:
    return None


def _rows(ref) -> int:
    n = 1
    for s in ref[1][:-1]:
        n *= int(s)
    return n


@dataclass
class Event:
    kind: str
    cmd_id: int
    stream: object = None
    cuda_event: object = None
    result: object = None
    error: BaseException | None = None
    finalize: object = None
    keep: object = None


class CudaBackend:
    device_side_waits = True

    def __init__(self, config: CudaBackendConfig) -> None:
        if config.allow_device_to_device:
            raise ValueError("device-to-device copies are not supported in Phase 1")
        if config.num_dpus <= 0:
            raise ValueError("num_dpus must be positive")
        if not torch.cuda.is_available():
            raise RuntimeError("CudaBackend needs a CUDA device (there is no CPU fallback)")
        self.config = config
        self.distributed = config.rank is not None
        if self.distributed:
            if not 0 <= config.rank < config.num_dpus:
                raise ValueError(f"rank {config.rank} outside [0, {config.num_dpus})")
            self.local = [config.rank]
            self._dev = {config.rank: torch.cuda.current_device()}
        else:
            devs = tuple(config.devices) if config.devices else (torch.cuda.current_device(),)
            self.local = list(range(config.num_dpus))
            self._dev = {d: devs[d % len(devs)] for d in self.local}
        self._arena = {}
        self._streams = {}
        for d in self.local:
            with torch.cuda.device(self._dev[d]):
                self._arena[d] = torch.zeros(config.mram_bytes_per_dpu, dtype=torch.uint8, device=self._dev[d])
                self._streams[d] = torch.cuda.Stream(self._dev[d])
        self.host_device = self._dev[self.local[0]]
        # With one local rank nothing can overlap its stream, so the host commands
        # share it: a plan is then one in-order chain with no cross-stream events.
        if len(self.local) == 1:
            self._host_stream = self._streams[self.local[0]]
        else:
            self._host_stream = torch.cuda.Stream(self.host_device)
        if not self.distributed:
            for a in set(self._dev.values()):
                for b in set(self._dev.values()):
                    if a != b:
                        nat.check(nat.lib.pim_enable_peer_access(a, b), "peer access")
        self._kernels: dict[str, object] = {}
        self._events: dict[int, Event] = {}
        # Per-plan state is keyed by id(plan) / id(cmd).  Every registered plan stays
        # referenced in _plans until release_plan, so no later object can reuse one of
        # those ids and pick up another plan's lowering.
        self._plans: dict[int, object] = {}
        self._lowered: dict[int, object] = {}
        self._host: dict[int, torch.Tensor] = {}
        self._scratch: dict[tuple, torch.Tensor] = {}
        self._err = {d: torch.zeros(4, dtype=torch.int32, device=self._dev[d]) for d in self.local}
        self._keep: list = []
        self._no_event: set[int] = set()
        self._capturing = False
        self._plan = None
        self.launches = 0
        self._p2p = None
        self.fused_allreduces = 0  # linear -> all_reduce -> add chains run as one kernel
        self.combine_adds = 0  # all_reduce -> add pairs run as one combine (combine_add)
        self.fused_attentions = 0  # attention commands computed inside their attn_in launch
        self.decode_layers = 0  # decode layers run as one pim_decode_layer launch
        self.decode_steps = 0  # decode plans run as one pim_decode_step launch
        if config.allreduce not in ("ordered", "p2p", "fused", "nccl"):
            raise ValueError(f"allreduce={config.allreduce!r}: expected ordered, p2p, fused or nccl")
        if self.distributed and config.allreduce in ("p2p", "fused"):
            from backend.p2p import P2PGroup

            with torch.cuda.device(self.host_device):
                self._p2p = P2PGroup.create(config.rank, config.num_dpus, self.host_device)
        for d in set(self._dev.values()):
            torch.cuda.synchronize(d)

    def close(self) -> None:
        """Finish queued work and release the arenas, workspaces and host buffers.

        NumpyBackend.close (backend/hal_numpy.py) shuts its worker pool down; here the
        device memory goes back to the caching allocator.  The backend is unusable after.
        """
        self.synchronize()
        if self._p2p is not None:
            self._p2p.close()
            self._p2p = None
        self._lowered.clear()
        self._plans.clear()
        self._events.clear()
        self._arena.clear()
        self._scratch.clear()
        self._host.clear()
        self._keep.clear()

    # -- addresses & streams ------------------------------------------------
    def arena(self, dpu_id: int) -> torch.Tensor:
        return self._arena[self._local(dpu_id)]

    def arena_ptr(self, dpu_id: int) -> int:
        return self.arena(dpu_id).data_ptr()

    def stream(self, dpu_id: int):
        return self._streams[self._local(dpu_id)]

    def stream_handle(self, dpu_id: int) -> int:
        return self.stream(dpu_id).cuda_stream

    def host_stream(self):
        return self._host_stream

    def host_stream_handle(self) -> int:
        return self._host_stream.cuda_stream

    def device_of(self, dpu_id: int) -> int:
        return self._dev[self._local(dpu_id)]

    def error_flag_ptr(self, dpu_id: int) -> int:
        return self._err[self._local(dpu_id)].data_ptr()

    def _local(self, dpu_id) -> int:
        d = int(dpu_id)
        if d not in self._arena:
            if 0 <= d < self.config.num_dpus:
                raise ValueError(f"dpu {d} is owned by another process (this process runs rank {self.local})")
            raise ValueError(f"dpu_id {d} out of range [0, {self.config.num_dpus})")
        return d

    def scratch(self, dpu_id: int, nbytes: int, pool=None) -> tuple[int, int]:
        """Per-rank kernel workspace, zero-filled and grow-only; returns (pointer, bytes).

        Commands that ask for the same ``pool`` share one buffer (they run in stream
        order on the rank).  The default pool holds data that no command expects to find
        again (normalised rows of a row batch); the attention kernel keeps per-row tickets
        that must read zero at every call, so each attention geometry has a pool of its
        own that nothing else writes.
        """
        if nbytes <= 0:
            return 0, 0
        d = self._local(dpu_id)
        key = (d, pool)
        cur = self._scratch.get(key)
        if cur is None or cur.numel() < nbytes:
            self.synchronize()
            cur = torch.zeros(int(nbytes), dtype=torch.uint8, device=self._dev[d])
            torch.cuda.synchronize(self._dev[d])
            if key in self._scratch:
                self._keep.append(self._scratch[key])  # earlier commands keep their pointer
            self._scratch[key] = cur
        return cur.data_ptr(), cur.numel()

    # -- NumpyBackend memory API ---------------------------------------------
    def _check(self, offset: int, nbytes: int) -> None:
        cap = self.config.mram_bytes_per_dpu
        if offset < 0 or nbytes < 0 or offset + nbytes > cap:
            raise ValueError(f"invalid MRAM range offset={offset} nbytes={nbytes} capacity={cap}")

    def copy_to_dpu(self, dpu_id: int, offset: int, data: np.ndarray) -> None:
        blob = np.ascontiguousarray(data).view(np.uint8).reshape(-1)
        self._check(offset, blob.nbytes)
        if self.distributed and int(dpu_id) not in self._arena:
            if not 0 <= int(dpu_id) < self.config.num_dpus:
                raise ValueError(f"dpu_id {dpu_id} out of range")
            return  # another process owns and loads that rank
        d = self._local(dpu_id)
        if blob.nbytes == 0:
            return
        st = self._streams[d]
        st.synchronize()
        with torch.cuda.stream(st):
            self._arena[d][offset:offset + blob.nbytes].copy_(torch.from_numpy(blob.copy()))
        st.synchronize()

    def copy_from_dpu(self, dpu_id: int, offset: int, shape, dtype) -> np.ndarray:
        dt = _np_dtype(dtype)
        n = int(np.prod(shape)) * dt.itemsize
        self._check(offset, n)
        d = self._local(dpu_id)
        self._streams[d].synchronize()
        self._host_stream.synchronize()
        with torch.cuda.stream(self._streams[d]):
            host = self._arena[d][offset:offset + n].cpu().numpy()
        return host.view(dt).reshape(shape).copy()

    def write_local(self, dpu_id: int, offset: int, data: np.ndarray) -> None:
        self.copy_to_dpu(dpu_id, offset, data)

    def read_local(self, dpu_id: int, offset: int, shape, dtype) -> np.ndarray:
        return self.copy_from_dpu(dpu_id, offset, shape, dtype)

    def push_xfer(self, transfers: list[tuple[int, int, np.ndarray]]) -> None:
        for dpu_id, offset, data in transfers:
            self.copy_to_dpu(dpu_id, offset, data)

    @property
    def dpu_set(self):
        """The reference exposes its SDK set here; on the B200 the ranks' arenas play that role."""
        return self

    # -- plans ----------------------------------------------------------------
    def register_kernel(self, name: str, fn) -> None:
        self._kernels[name] = fn

    def _allreduce_fusions(self, plan) -> dict:
        """Chains ``linear`` -> all_reduce combine -> ``add`` of this rank to run as one kernel.

        One process per GPU with a P2P group: the row-parallel projection writes its
        partial into every rank's exchange buffer and the same kernel produces the add's
        output (``lower_linear_allreduce``).  A chain qualifies when the edge is a plain
        rank-order sum of one full-tensor segment per rank that fits the exchange rows,
        nothing reads the sum on the host, the linear (the last one before the combine
        that writes the collected range) has at most 8 rows, the first ``add`` after the
        combine that reads the sum takes it, and no command between the linear and the
        add (other than
        the edge's own transfers, which the fused kernel replaces) touches the add's
        output (or the sum's destination, when something besides the add reads the sum)
        or writes the add's other input.  Returns {linear id: (linear, combine, add, sum
        offset read by the add, sum offset to write or None)}.
        """
        g = self._p2p
        if g is None or self.config.allreduce != "fused":
            return {}
        me = self.local[0]
        cmds = plan.commands
        pos = {c.id: i for i, c in enumerate(cmds)}
        host_bytes = self._host[id(plan)].numel()

        def launch_of(c, kernel):
            return c.op == "launch" and c.dpu_id == me and c.payload.get("kernel") == kernel
        out = {}
        for c in cmds:
            if c.payload.get("role") != "combine" or c.payload.get("kind") != "all_reduce":
                continue
            e = c.payload["entry"]
            nbytes = e.numel * e.dtype.itemsize
            mine = [s for s in e.collect_segments if s.src_dpu == me]
            wb = [s for s in e.writeback_segments if s.dst_dpu == me]
            if (e.reduce == "mean" or [s.src_dpu for s in e.collect_segments] != list(range(g.size))
                    or len(mine) != 1 or mine[0].nbytes != nbytes or len(wb) != 1 or wb[0].nbytes != nbytes
                    or not g.fits(nbytes) or c.payload["host_offset"] < host_bytes):
                continue
            lin = next((m for m in reversed(cmds[:pos[c.id]])
                        if launch_of(m, "linear") and m.payload["output"][0] == mine[0].src_addr), None)
            add = next((m for m in cmds[pos[c.id] + 1:]
                        if launch_of(m, "add") and any(r[0] == wb[0].dst_addr for r in m.payload["inputs"])), None)
            if lin is None or add is None or _rows(lin.payload["inputs"][0]) > 8:
                continue
            res = [r for r in add.payload["inputs"] if r[0] != wb[0].dst_addr]
            if len(res) != 1:
                continue
            loc = ("dpu", me)
            y = Access(loc, add.payload["output"][0], nbytes)
            r_acc = Access(loc, res[0][0], nbytes)
            s_acc = Access(loc, wb[0].dst_addr, nbytes)
            edge = c.payload.get("edge")
            sum_read = _read_before_overwritten(cmds[pos[c.id] + 1:], me, s_acc, skip=add, edge=edge)
            touched = [y, s_acc] if sum_read else [y]
            if _window_clear(cmds[pos[lin.id] + 1:pos[add.id]], me, touched, [r_acc], edge=edge):
                out[lin.id] = (lin, c, add, wb[0].dst_addr, wb[0].dst_addr if sum_read else None)
        return out

    def _combine_add_fusions(self, plan) -> dict:
        """All_reduce combines whose consuming residual ``add`` runs inside the combine.

        One process per GPU, ``allreduce="ordered"`` or ``"p2p"`` and ``combine_add``: the edge is a plain
        rank-order sum of one full-tensor segment per rank with no host reader (and below
        the split threshold), the first ``add`` of this rank after the combine reads the
        sum, and no command between the combine and that add (other than the edge's own
        transfers) touches the add's output (or the sum's destination, when something
        besides the add reads the sum) or writes the add's other input.  Returns {combine
        id: (add, residual offset, output offset, sum offset to write or None)}.
        """
        cfg = self.config
        if not self.distributed or cfg.allreduce not in ("ordered", "p2p") or not cfg.combine_add:
            return {}
        me = self.local[0]
        cmds = plan.commands
        pos = {c.id: i for i, c in enumerate(cmds)}
        host_bytes = self._host[id(plan)].numel()
        out = {}
        for c in cmds:
            if c.payload.get("role") != "combine" or c.payload.get("kind") != "all_reduce":
                continue
            e = c.payload["entry"]
            nbytes = e.numel * e.dtype.itemsize
            mine = [s for s in e.collect_segments if s.src_dpu == me]
            wb = [s for s in e.writeback_segments if s.dst_dpu == me]
            order = [s.src_dpu for s in e.collect_segments]
            if (e.reduce == "mean" or sorted(order) != list(range(cfg.num_dpus)) or len(mine) != 1
                    or mine[0].nbytes != nbytes or len(wb) != 1 or wb[0].nbytes != nbytes
                    or c.payload["host_offset"] < host_bytes
                    or (cfg.allreduce_split_bytes and nbytes >= cfg.allreduce_split_bytes)):
                continue
            add = next((m for m in cmds[pos[c.id] + 1:]
                        if m.op == "launch" and m.dpu_id == me and m.payload.get("kernel") == "add"
                        and any(r[0] == wb[0].dst_addr for r in m.payload["inputs"])), None)
            if add is None or add.payload["output"][2] != e.dtype.name:
                continue
            res = [r for r in add.payload["inputs"] if r[0] != wb[0].dst_addr]
            if len(res) != 1 or _rows(res[0]) * res[0][1][-1] != e.numel:
                continue
            loc = ("dpu", me)
            y = Access(loc, add.payload["output"][0], nbytes)
            r_acc = Access(loc, res[0][0], nbytes)
            s_acc = Access(loc, wb[0].dst_addr, nbytes)
            edge = c.payload.get("edge")
            sum_read = _read_before_overwritten(cmds[pos[c.id] + 1:], me, s_acc, skip=add, edge=edge)
            touched = [y, s_acc] if sum_read else [y]
            if _window_clear(cmds[pos[c.id] + 1:pos[add.id]], me, touched, [r_acc], edge=edge):
                out[c.id] = (add, res[0][0], add.payload["output"][0], wb[0].dst_addr if sum_read else None)
        return out

    def _attention_fusions(self, plan) -> dict:
        """Decode ``attention`` commands computed inside the preceding ``attn_in`` launch.

        With ``fuse_attention``, per local rank: the attention reads the q that an
        ``attn_in`` of the same rank wrote, the same layer's KV blocks and positions, has at
        most 8 query rows, 1-64 heads of dimension 64 or 128, and no command between the two
        (other than on other ranks) touches the attention's output or writes the q, the
        positions or the layer's KV.  Returns {attn_in id: attention command}.
        """
        if not self.config.fuse_attention:
            return {}
        cmds = plan.commands
        out = {}
        last_in: dict[int, int] = {}  # rank -> index of its latest attn_in
        for idx, c in enumerate(cmds):
            if c.op != "launch" or c.dpu_id is None or int(c.dpu_id) not in self._arena:
                continue
            k = c.payload.get("kernel")
            if k == "attn_in":
                last_in[int(c.dpu_id)] = idx
                continue
            if k != "attention" or int(c.dpu_id) not in last_in:
                continue
            d = int(c.dpu_id)
            ai = cmds[last_in[d]]
            q, pos = c.payload["inputs"]
            out_off, out_shape, out_dt = c.payload["output"]
            hd = c.payload["kv"]["head_dim"]
            rows = _rows(q)
            hq = q[1][-1] // hd if hd else 0
            if (ai.payload["output"][0] != q[0] or ai.payload["inputs"][5][0] != pos[0]
                    or ai.payload["kv"]["layer_base"] != c.payload["kv"]["layer_base"] or rows > 8
                    or hd not in (64, 128) or not 1 <= hq <= 64 or out_dt != q[2]):
                continue
            loc = ("dpu", d)
            nbytes = _rows(c.payload["output"]) * out_shape[-1] * _ITEM.get(out_dt, 4)
            o_acc = Access(loc, out_off, nbytes)
            written = [Access(loc, q[0], rows * q[1][-1] * _ITEM.get(q[2], 4))]
            written += [a for a in ai.writes if a.loc == loc]  # the layer's KV blocks
            # attn_in's CTAs still read its inputs while the first heads' outputs are written
            if any(r.overlaps(o_acc) for r in ai.reads):
                continue
            if _window_clear(cmds[last_in[d] + 1:idx], d, [o_acc], written, host_writes=True):
                out[ai.id] = c
        return out

    def _decode_layer_fusions(self, plan, fused=None) -> dict:
        """Decode layers run as one ``pim_decode_layer`` launch.

        With ``decode_layer``, per local rank, on the commands that do something on that
        rank (its launches and the host commands; the transfers, combines and adds of the
        ``fused`` all-reduce chains of ``_allreduce_fusions`` left out): five consecutive
        commands attn_in, attention, o_proj, mlp_in, down_proj where each reads the
        previous one's output (the attention the attn_in's q, positions and KV blocks).
        One rank in all (TP = 1): o_proj and down_proj are ``linear_add`` launches.  One
        process per GPU in ``allreduce="fused"`` mode: they are ``linear`` launches that
        head fused all-reduce chains, whose adds' outputs the next phase reads.  One
        activation row of one sequence, 1-64 query heads of dimension 64 or 128, one
        dtype, rows of a multiple of 16 bytes and activations of at most 96 KB.  The
        attention's output must not overlap what attn_in reads (the first heads are
        written while other CTAs still read the layer's input).  Returns {attn_in id:
        (the five commands, the two all-reduce chains or None)}.
        """
        cfg = self.config
        fused = fused or {}
        if not (cfg.decode_layer or getattr(cfg, "decode_step", False)):
            return {}
        if cfg.num_dpus == 1 and not self.distributed:
            ar, kinds = False, ("attn_in", "attention", "linear_add", "mlp_in", "linear_add")
        elif self.distributed and fused:
            ar, kinds = True, ("attn_in", "attention", "linear", "mlp_in", "linear")
        else:
            return {}
        skip = {id(f[1]) for f in fused.values()} | {id(f[2]) for f in fused.values()}
        edges = {f[1].payload.get("edge") for f in fused.values()}
        out = {}
        for me in self.local:
            seq = [c for c in plan.commands
                   if _on_rank(c, me) and id(c) not in skip
                   and not (c.payload.get("role") in ("collect", "writeback") and c.payload.get("edge") in edges)]
            for i in range(len(seq) - 4):
                chain = seq[i:i + 5]
                if any(c.op != "launch" or c.dpu_id is None or c.payload.get("kernel") != k
                       for c, k in zip(chain, kinds)):
                    continue
                if ar and (chain[2].id not in fused or chain[4].id not in fused):
                    continue
                ai, at, o, mi, dn = (c.payload for c in chain)
                # the outputs the next phases read: at TP > 1 the fused chains' add outputs
                o_out = fused[chain[2].id][2].payload["output"] if ar else o["output"]
                dn_out = fused[chain[4].id][2].payload["output"] if ar else dn["output"]
                x, q = ai["inputs"][0], at["inputs"][0]
                kv = ai["kv"]
                hd = kv["head_dim"]
                dts = {c.payload["inputs"][0][2] for c in chain} | {o_out[2], dn_out[2]}
                if len(dts) != 1 or next(iter(dts)) not in ("bfloat16", "float32"):
                    continue
                item = _ITEM[x[2]]
                hq = q[1][-1] // hd if hd else 0
                if (_rows(x) != 1 or x[1][1] != 1 or hd not in (64, 128) or not 1 <= hq <= 64
                        or hq % len(kv["kv_heads"]) or q[0] != ai["output"][0]
                        or at["inputs"][1][0] != ai["inputs"][5][0] or at["kv"]["layer_base"] != kv["layer_base"]):
                    continue
                if (o["inputs"][0][0] != at["output"][0] or mi["inputs"][0][0] != o_out[0]
                        or dn["inputs"][0][0] != mi["output"][0]):
                    continue
                ks = [c.payload["inputs"][0][1][-1] for c in chain if c.payload["kernel"] != "attention"]
                # x, norm weight and weight of each projection start on 16 bytes
                offs = [r[0] for c in (ai, mi) for r in c["inputs"][:3]]
                offs += [r[0] for c in (o, dn) for r in c["inputs"][:2]]
                if any(k * item % 16 or k * item > 96 * 1024 for k in ks) or any(off % 16 for off in offs):
                    continue
                o_acc = Access(("dpu", me), at["output"][0], q[1][-1] * item)
                if any(r.overlaps(o_acc) for r in chain[0].reads):
                    continue
                out[chain[0].id] = (tuple(chain), (fused[chain[2].id], fused[chain[4].id]) if ar else None)
        return out

    def _decode_step_fusion(self, plan, fused, layers) -> dict:
        """With ``decode_step`` (and the conditions of ``decode_layer``): when the rank's
        working commands (as in ``_decode_layer_fusions``) hold a run of fused layers back
        to back, each reading the previous one's output, followed at once by the
        ``lm_head_in`` that reads the last layer's output, the run and the head are one
        launch.  Returns {first attn_in id: ([(chain, all-reduces) per layer], lm_head_in)}.
        """
        if not self.config.decode_step or not layers:
            return {}
        fused = fused or {}
        skip = {id(f[1]) for f in fused.values()} | {id(f[2]) for f in fused.values()}
        edges = {f[1].payload.get("edge") for f in fused.values()}
        out = {}
        for me in self.local:
            seq = [c for c in plan.commands
                   if _on_rank(c, me) and id(c) not in skip
                   and not (c.payload.get("role") in ("collect", "writeback") and c.payload.get("edge") in edges)]
            i = 0
            while i < len(seq):
                if seq[i].id not in layers:
                    i += 1
                    continue
                run, j = [], i
                while j < len(seq) and seq[j].id in layers:
                    chain, ar = layers[seq[j].id]
                    if seq[j:j + 5] != list(chain):
                        break
                    if run:  # reads the previous layer's output
                        prev_chain, prev_ar = run[-1]
                        prev_out = prev_ar[1][2].payload["output"][0] if prev_ar else prev_chain[4].payload["output"][0]
                        if chain[0].payload["inputs"][0][0] != prev_out:
                            break
                    run.append((chain, ar))
                    j += 5
                head = seq[j] if j < len(seq) else None
                if run and head is not None and head.op == "launch" and head.payload.get("kernel") == "lm_head_in":
                    last_chain, last_ar = run[-1]
                    last_out = last_ar[1][2].payload["output"] if last_ar else last_chain[4].payload["output"]
                    x = head.payload["inputs"][0]
                    if (x[0] == last_out[0] and _rows(x) == 1 and x[2] == last_out[2]
                            and all(r[0] % 16 == 0 for r in head.payload["inputs"][:3])):
                        out[run[0][0][0].id] = (run, head)
                i = max(j, i + 1)
        return out

    def register_plan(self, plan) -> None:
        from backend.cuda_collectives import lower_combine
        from backend.cuda_kernels import lower_decode_layer, lower_decode_step, lower_linear_allreduce

        self._plans[id(plan)] = plan
        layout = plan.meta.get("host_layout")
        size = max(layout.total if layout else 0, 256)
        self._host[id(plan)] = torch.zeros(size, dtype=torch.uint8, device=self.host_device)
        fused = self._allreduce_fusions(plan)
        absorbed = {id(f[1]) for f in fused.values()} | {id(f[2]) for f in fused.values()}
        self.fused_allreduces += len(fused)
        comb_add = self._combine_add_fusions(plan) if not fused else {}
        absorbed |= {id(f[0]) for f in comb_add.values()}
        self.combine_adds += len(comb_add)
        layers = self._decode_layer_fusions(plan, fused)
        absorbed |= {id(c) for ch, _ in layers.values() for c in ch[1:]}
        self.decode_layers += len(layers)
        steps = self._decode_step_fusion(plan, fused, layers)
        for run, head in steps.values():  # the layers after the first, and the head, join the step launch
            absorbed |= {id(c) for chain, _ in run[1:] for c in chain} | {id(head)}
        self.decode_steps += len(steps)
        attn = self._attention_fusions(plan) if not layers else {}
        absorbed |= {id(c) for c in attn.values()}
        self.fused_attentions += len(attn)
        for cmd in plan.commands:
            role = cmd.payload.get("role")
            if id(cmd) in absorbed:
                self._lowered[id(cmd)] = _noop  # done by the fused projection kernel
            elif cmd.id in steps:
                self._lowered[id(cmd)] = lower_decode_step(self, cmd.dpu_id, *steps[cmd.id])
            elif cmd.id in layers:
                self._lowered[id(cmd)] = lower_decode_layer(self, cmd.dpu_id, *layers[cmd.id])
            elif cmd.id in fused:
                lin, _, add, sum_in_add, sum_off = fused[cmd.id]
                self._lowered[id(cmd)] = lower_linear_allreduce(self, cmd.dpu_id, lin, add, sum_in_add, sum_off)
            elif cmd.op == "launch" and cmd.payload.get("kernel") not in self._kernels:
                if cmd.dpu_id in self._arena:
                    self._lowered[id(cmd)] = lower_launch(self, cmd.dpu_id, cmd, attn_fusion=attn.get(cmd.id))
            elif role == "combine":
                self._lowered[id(cmd)] = lower_combine(self, plan, cmd, add_fusion=comb_add.get(cmd.id))
            elif cmd.op == "host_op":
                self._lowered[id(cmd)] = lower_host_op(self, plan, cmd)
        # A command needs a recorded CUDA event only when a command on another stream
        # waits for it; leaving the others unrecorded keeps consecutive kernels of a
        # rank back to back in the stream (and in a captured graph), so programmatic
        # dependent launch can overlap them.
        def stream_key(c):
            s = self._host_stream if c.dpu_id is None else self._streams.get(int(c.dpu_id))
            return id(s) if s is not None else ("remote", c.dpu_id)

        stream_of = {c.id: stream_key(c) for c in plan.commands}
        needed = set()
        for c in plan.commands:
            for w in c.waits:
                if stream_of.get(w) != stream_of[c.id]:
                    needed.add(w)
        for c in plan.commands:
            if c.id not in needed and c.payload.get("fn") is None:
                self._no_event.add(id(c))
        for d in set(self._dev.values()):
            torch.cuda.synchronize(d)  # descriptor tables and host arena were written on the default stream
        self._plan = plan

    def release_plan(self, plan) -> None:
        """Drop a registered plan's host buffer and lowered commands (after its queued work
        and every graph captured from it are finished).  A plan must be registered again
        before it runs after this."""
        if self._plans.pop(id(plan), None) is None:
            return
        self.synchronize()
        for cmd in plan.commands:
            self._lowered.pop(id(cmd), None)
            self._no_event.discard(id(cmd))
        self._host.pop(id(plan), None)
        if self._plan is plan:
            self._plan = None

    def host_ptr(self, plan) -> int:
        return self._host[id(plan)].data_ptr()

    def host_tensor(self, plan) -> torch.Tensor:
        return self._host[id(plan)]

    def write_host(self, plan, offset: int, data: np.ndarray) -> None:
        blob = np.ascontiguousarray(data).view(np.uint8).reshape(-1)
        buf = self._host[id(plan)]
        if offset < 0 or offset + blob.nbytes > buf.numel():
            raise ValueError(f"invalid host range offset={offset} nbytes={blob.nbytes}")
        self.synchronize()  # graph replays run on a rank stream; order after everything
        with torch.cuda.stream(self._host_stream):
            buf[offset:offset + blob.nbytes].copy_(torch.from_numpy(blob.copy()))
        self._host_stream.synchronize()

    def read_host(self, plan, offset: int, shape, dtype) -> np.ndarray:
        dt = _np_dtype(dtype)
        n = int(np.prod(shape)) * dt.itemsize
        self.synchronize()
        with torch.cuda.stream(self._host_stream):
            host = self._host[id(plan)][offset:offset + n].cpu().numpy()
        return host.view(dt).reshape(shape).copy()

    def begin_run(self, plan=None) -> None:
        """Clear the command-id table and order every stream after all earlier work (device side)."""
        self._events.clear()
        if plan is not None:
            self._plan = plan
        if self._capturing:
            # inside a capture only fork the other streams from the capture origin
            origin = self.capture_stream()
            e = torch.cuda.Event()
            e.record(origin)
            for s in self._all_streams():
                if s is not origin:
                    s.wait_event(e)
            return
        streams = self._all_streams()
        marks = []
        for s in streams:
            e = torch.cuda.Event()
            e.record(s)
            marks.append((s, e))
        for s in streams:
            for s2, e in marks:
                if s2 is not s:
                    s.wait_event(e)

    def _all_streams(self) -> list:
        out = [self._streams[d] for d in self.local]
        return out if self._host_stream in out else out + [self._host_stream]

    def capture_stream(self):
        """Origin stream of graph capture and replay: the first local rank's stream.

        The rank stream carries the long chain of kernels; capturing it as the
        origin (the host stream and other ranks fork from it and join back) keeps
        its consecutive kernels connected by programmatic-launch edges in the graph.
        """
        return self._streams[self.local[0]]

    def end_run(self) -> None:
        """Join every other stream into the capture origin (used when capturing a plan)."""
        origin = self.capture_stream()
        for s in self._all_streams():
            if s is not origin:
                e = torch.cuda.Event()
                e.record(s)
                origin.wait_event(e)

    # -- async core -------------------------------------------------------------
    def submit(self, cmd) -> Event:
        if cmd.id in self._events:
            raise ValueError(f"duplicate command id {cmd.id}")
        deps = []
        for w in cmd.waits:
            ev = self._events.get(w)
            if ev is None:
                raise ValueError(f"unknown dependency command id {w}")
            deps.append(ev)
        kind = "dpu" if cmd.op == "launch" else ("dma" if cmd.op in ("dma_in", "dma_out") else "host")
        if cmd.dpu_id is not None and self.distributed and int(cmd.dpu_id) not in self._arena:
            ev = Event(kind, cmd.id)  # runs in the process that owns that rank
            self._events[cmd.id] = ev
            return ev
        if cmd.dpu_id is not None and not 0 <= int(cmd.dpu_id) < self.config.num_dpus:
            ev = Event(kind, cmd.id, error=ValueError(f"dpu_id {cmd.dpu_id} out of range"))
            self._events[cmd.id] = ev
            return ev
        stream = self._streams[int(cmd.dpu_id)] if cmd.dpu_id is not None else self._host_stream
        ev = Event(kind, cmd.id, stream)
        fn = cmd.payload.get("fn")
        if cmd.dpu_id is None and callable(fn) and id(cmd) not in self._lowered:
            # host callable of the HAL API: runs on the host after its dependencies
            for dep in deps:
                if dep.cuda_event is not None:
                    dep.cuda_event.synchronize()
            try:
                ev.result = fn(cmd)
            except BaseException as exc:  # surfaces at wait, like a failed future
                ev.error = exc
            ev.stream = None
            self._events[cmd.id] = ev
            return ev
        for dep in deps:
            if dep.cuda_event is not None and dep.stream is not stream:
                stream.wait_event(dep.cuda_event)
        try:
            self._enqueue(cmd, stream, ev)
        except BaseException as exc:
            ev.error = exc
        if id(cmd) not in self._no_event or ev.finalize is not None:
            e = torch.cuda.Event()
            e.record(stream)
            ev.cuda_event = e
        self._events[cmd.id] = ev
        return ev

    def _enqueue(self, cmd, stream, ev: Event) -> None:
        p = cmd.payload
        role = p.get("role")
        low = self._lowered.get(id(cmd))
        if low is not None:
            low()
            self.launches += 1
            return
        if cmd.op == "launch":
            fn = self._kernels.get(str(p.get("kernel")))
            if fn is None:
                raise KeyError(f"no kernel registered for {p.get('kernel')!r}")
            with torch.cuda.stream(stream):
                fn(self, int(cmd.dpu_id), cmd)
            return
        if role in ("collect", "writeback"):
            return  # the edge's data moves inside its combine command
        if cmd.op == "dma_in":
            data = np.ascontiguousarray(np.asarray(p["data"])).copy()
            blob = data.view(np.uint8).reshape(-1)
            off = int(p["offset"])
            self._check(off, blob.nbytes)
            src = torch.from_numpy(blob).pin_memory()
            ev.keep = src
            with torch.cuda.stream(stream):
                self._arena[int(cmd.dpu_id)][off:off + blob.nbytes].copy_(src, non_blocking=True)
            return
        if cmd.op == "dma_out":
            dt = _np_dtype(p["dtype"])
            shape = tuple(p["shape"])
            n = int(np.prod(shape)) * dt.itemsize
            off = int(p["offset"])
            self._check(off, n)
            dst = torch.empty(n, dtype=torch.uint8, pin_memory=True)
            with torch.cuda.stream(stream):
                dst.copy_(self._arena[int(cmd.dpu_id)][off:off + n], non_blocking=True)
            ev.keep = dst
            ev.finalize = lambda: dst.numpy().copy().view(dt).reshape(shape)
            return
        if cmd.dpu_id is None:
            return
        raise ValueError(f"unsupported command op {cmd.op!r}")

    def wait(self, event: Event, timeout: float | None = None):
        if event.error is not None:
            raise event.error
        if event.cuda_event is None and event.stream is not None:
            # unrecorded plan command: everything enqueued so far on its stream covers it
            event.cuda_event = torch.cuda.Event()
            event.cuda_event.record(event.stream)
        if event.cuda_event is not None:
            if timeout is None:
                event.cuda_event.synchronize()
            else:
                deadline = time.monotonic() + timeout
                while not event.cuda_event.query():
                    if time.monotonic() > deadline:
                        raise TimeoutError(f"command {event.cmd_id} did not complete within {timeout}s")
                    time.sleep(20e-6)
        if event.finalize is not None:
            event.result = event.finalize()
            event.finalize = None
        return event.result

    def query(self, event: Event) -> bool:
        if event.error is not None:
            return True
        if event.cuda_event is None:
            return True if event.stream is None else bool(event.stream.query())
        return bool(event.cuda_event.query())

    def synchronize(self) -> None:
        for s in self._streams.values():
            s.synchronize()
        self._host_stream.synchronize()

    def read_error_flags(self) -> dict[int, int]:
        """Per local rank, the first non-zero device error word (0 when none was raised).

        Words: 0 embedding id out of range, 1 a projection kernel's bounded wait, 2 a
        peer all-reduce's bounded wait for another rank, 3 a decode-layer grid barrier's
        bounded wait.
        """
        self.synchronize()
        out = {}
        for d, t in self._err.items():
            words = [int(v) for v in t.tolist()]
            out[d] = next((w for w in words if w), 0)
        return out

    # -- CUDA graphs ---------------------------------------------------------------
    def capture(self, plan) -> "CapturedPlan":
        """Record one execution of ``plan`` into a CUDA graph; inputs are read from device buffers."""
        from runtime.executor import execute_plan

        execute_plan(plan, self, sync=True)  # warm-up: lazy initialisation outside the capture
        self.synchronize()
        g = torch.cuda.CUDAGraph()
        self._capturing = True
        n0 = nat.lib.pim_kernel_launches()
        try:
            with torch.cuda.device(self.device_of(self.local[0])):
                with torch.cuda.graph(g, stream=self.capture_stream(), capture_error_mode="relaxed"):
                    execute_plan(plan, self, sync=False)
                    self.end_run()
        finally:
            self._capturing = False
        self._events.clear()
        return CapturedPlan(self, plan, g, kernels=int(nat.lib.pim_kernel_launches() - n0))


@dataclass
class CapturedPlan:
    hal: CudaBackend
    plan: object
    graph: object
    kernels: int = 0  # kernels of this library recorded in the graph (launched by every replay)
    replays: int = field(default=0)

    def replay(self) -> None:
        """Launch the graph on the capture-origin stream (ordered after earlier work there)."""
        with torch.cuda.stream(self.hal.capture_stream()):
            self.graph.replay()
        self.replays += 1
