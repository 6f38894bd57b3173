"""Column-parallel quantized matmul over several GPUs (one process per GPU).

The reference quantizes each output column independently (one scale per
column, src/quantization/quantization.cpp:141-159) and stores a column's codes
contiguously (quantization.cpp:155), so a weight splits into column shards
with no communication: rank r owns columns [begin_r, end_r), computes
y[:, begin_r:end_r] = matmul(x, W[:, begin_r:end_r]) with the same
activation codes as every other rank (the per-row quantizer depends only on
x), and the shards are joined with one NCCL all-gather only when the caller
needs the full output.  Results are bit-identical to the single-GPU matmul.
"""
from __future__ import annotations


def column_ranges(n_cols: int, world: int):
    """Contiguous, balanced column shards: the first n_cols % world ranks get
    one extra column."""
    if world < 1:
        raise ValueError("world must be >= 1")
    if n_cols < world:
        raise ValueError(f"cannot split {n_cols} columns over {world} ranks")
    base, extra = divmod(n_cols, world)
    out, c = [], 0
    for r in range(world):
        w = base + (1 if r < extra else 0)
        out.append((c, c + w))
        c += w
    return out


def shard_weight(weight, rank: int, world: int):
    """This rank's column shard of a QuantizedMatrix (device to device)."""
    b, e = column_ranges(weight.cols(), world)[rank]
    return weight.slice_cols(b, e)


def assemble_columns(blocks, ranges, out=None):
    """Join gathered per-rank blocks [M, n_r] into [M, N] (column order of
    ``ranges``)."""
    import torch

    M = blocks[0].shape[0]
    N = ranges[-1][1]
    if out is None:
        out = torch.empty((M, N), dtype=blocks[0].dtype, device=blocks[0].device)
    for (b, e), blk in zip(ranges, blocks):
        out[:, b:e].copy_(blk)
    return out


def sharded_matmul(x, weight_shard, n_cols: int, group=None, gather: bool = True, matmul_fn=None, bias_shard=None):
    """y = matmul(x, W) with W column-sharded over the process group.

    ``weight_shard`` is this rank's shard (see :func:`shard_weight`),
    ``n_cols`` the full column count.  With ``gather`` every rank returns the
    full [M, n_cols] output (one all-gather), otherwise its own block.
    ``matmul_fn`` defaults to :func:`zyron_b200.quantization.matmul`.
    """
    import torch
    import torch.distributed as dist

    if matmul_fn is None:
        from .quantization import matmul as matmul_fn
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    ranges = column_ranges(n_cols, world)
    local = matmul_fn(x, weight_shard, bias=bias_shard) if bias_shard is not None else matmul_fn(x, weight_shard)
    b, e = ranges[rank]
    if local.shape[-1] != e - b:
        raise ValueError(f"rank {rank}: shard has {local.shape[-1]} columns, expected {e - b}")
    if not gather or world == 1:
        return local
    widths = [e - b for b, e in ranges]
    M = local.shape[0]
    wmax = max(widths)
    send = local.contiguous()
    if send.shape[1] != wmax:  # uneven split: pad this block to the widest shard
        send = torch.nn.functional.pad(send, (0, wmax - send.shape[1]))
    buf = torch.empty((world * M, wmax), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(buf, send, group=group)
    blocks = [blk[:, :w] for blk, w in zip(buf.view(world, M, wmax).unbind(0), widths)]
    return assemble_columns(blocks, ranges)


class PeerOutputs:
    """Full [rows, cols] fp32 outputs on every rank of the process group, each
    rank holding device pointers to all the others' copies (CUDA IPC handles
    from ``zq_ipc_export``, opened with ``zq_ipc_import`` while this rank's
    device is current, so its kernels reach them over NVLink).

    ``sharded_matmul_gathered`` lets the matmul epilogue store every output
    tile straight into all these buffers (``zq_matmul_multi``), so the
    all-gather of column-sharded outputs happens inside the matmul.

    There are ``buffers`` sets of outputs (default 2), used in turn: the
    output of one call stays intact while the next call runs, and is
    overwritten by the call after that.
    """

    def __init__(self, rows, cols, device, group=None, buffers=2):
        import ctypes as C

        import torch
        import torch.distributed as dist

        from . import _lib

        if buffers < 1:
            raise ValueError("buffers must be >= 1")
        L = _lib.lib()
        self.rows, self.cols = rows, cols
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.buffers = [torch.empty((rows, cols), dtype=torch.float32, device=device) for _ in range(buffers)]
        self._imported = []
        self._pointers = []
        for buf in self.buffers:
            h = _lib.IpcHandle()
            _lib.check(L.zq_ipc_export(C.c_void_p(buf.data_ptr()), C.byref(h)))
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(h), group=group)
            # import the peers' buffers with this rank's device current, so the
            # matmul running here may store into them (peer access over NVLink)
            peers = []
            with torch.cuda.device(device):
                for r, raw in enumerate(handles):
                    if r == self.rank:
                        continue
                    ph = _lib.IpcHandle.from_buffer_copy(raw)
                    p = C.c_void_p()
                    _lib.check(L.zq_ipc_import(C.byref(ph), C.byref(p)))
                    peers.append(p.value)
            self._imported += peers
            # destination order: own buffer first, then the peers
            self._pointers.append([buf.data_ptr()] + peers)
        self.turn = 0  # the buffer set the next call writes
        self.local = self.buffers[0]  # the last call's output on this rank
        self._flag = torch.zeros(1, dtype=torch.float32, device=device)

    @property
    def pointers(self):
        """Destinations of the next call: this rank's buffer, then the peers'."""
        return self._pointers[self.turn]

    def close(self):
        from . import _lib

        for p in self._imported:
            _lib.lib().zq_ipc_close(p)
        self._imported = []
        self._pointers = []

    def barrier(self):
        """Stream-ordered barrier: completes (on the stream) once every rank's
        stream has reached it."""
        import torch.distributed as dist

        dist.all_reduce(self._flag, group=self.group)


def sharded_matmul_gathered(x, weight_shard, peer_out: PeerOutputs, bias_shard=None, workspace=None, stream=None):
    """y = matmul(x, W) with W column-sharded over the group; every rank ends
    with the full [M, N] output.  The matmul epilogue writes each tile to all
    ranks' outputs over NVLink; no separate collective moves the data.

    Ordering, on the stream of the call (all ranks must make the same calls
    in the same order):
      - a barrier before the matmul: no rank stores into a peer's buffer
        until every rank's stream has reached this call, so work the peers
        queued before it (reads of older outputs) has finished;
      - a barrier after it: every rank's stores into this rank's output have
        landed when the returned tensor is read on the stream.
    The returned tensor is one of ``peer_out.buffers``, reused in turn: it
    holds this call's result until this rank issues the call after next
    (with the default two buffers).  Reads of it on another stream must be
    ordered with this one."""
    import ctypes as C

    import torch

    from . import _lib
    from .quantization import workspace as get_workspace

    L = _lib.lib()
    ranges = column_ranges(peer_out.cols, peer_out.world)
    b, e = ranges[peer_out.rank]
    if weight_shard.cols() != e - b:
        raise ValueError("weight shard does not match this rank's column range")
    x = x.contiguous()
    m = x.shape[0]
    s = stream if stream is not None else torch.cuda.current_stream(x.device)
    ws, ws_bytes = workspace if workspace is not None else get_workspace(weight_shard, m, x.device, s.cuda_stream)
    turn = peer_out.turn
    dst = peer_out.pointers
    ptrs = (C.c_void_p * len(dst))(*dst)
    with torch.cuda.stream(s):
        peer_out.barrier()
        _lib.check(L.zq_matmul_multi(weight_shard.handle, C.c_void_p(x.data_ptr()), m,
                                     None if bias_shard is None else C.c_void_p(bias_shard.data_ptr()),
                                     ptrs, len(dst), peer_out.cols, b, C.c_void_p(ws), ws_bytes,
                                     C.c_void_p(s.cuda_stream)))
        peer_out.barrier()
    peer_out.turn = (turn + 1) % len(peer_out.buffers)
    peer_out.local = peer_out.buffers[turn]
    return peer_out.local


_NCCL_ID_BYTES = 128  # ZQ_NCCL_UNIQUE_ID_BYTES


class NcclComm:
    """An NCCL communicator made by the library (``zq_nccl_comm_init``) over
    the ranks of a torch.distributed group, for :func:`nccl_sharded_matmul`.
    Rank 0 creates the unique id and the group (any backend) broadcasts it.
    Without an initialised process group it is a single-rank communicator."""

    def __init__(self, device, group=None):
        import ctypes as C

        import torch
        import torch.distributed as dist

        from . import _lib

        self._L = _lib.lib()
        if dist.is_initialized():
            self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        else:
            self.world, self.rank = 1, 0
        uid = (C.c_ubyte * _NCCL_ID_BYTES)()
        if self.rank == 0:
            _lib.check(self._L.zq_nccl_get_unique_id(uid))
        if self.world > 1:
            obj = [bytes(uid)]
            src = 0 if group is None else dist.get_global_rank(group, 0)
            dist.broadcast_object_list(obj, src=src, group=group)
            uid = (C.c_ubyte * _NCCL_ID_BYTES).from_buffer_copy(obj[0])
        self.handle = C.c_void_p()
        with torch.cuda.device(device):
            _lib.check(self._L.zq_nccl_comm_init(self.world, uid, self.rank, C.byref(self.handle)))

    def close(self):
        if self.handle:
            from . import _lib

            _lib.check(self._L.zq_nccl_comm_destroy(self.handle))
            self.handle = None


def nccl_sharded_matmul(x, weight_shard, n_cols: int, comm: NcclComm, bias_shard=None, out=None, stream=None):
    """y = matmul(x, W) with W column-sharded over ``comm``'s ranks, through
    the C entry point ``zq_matmul_sharded``: each rank computes its block of
    :func:`column_ranges` columns, one NCCL all-gather joins the blocks, and
    every rank returns the full [M, n_cols] output (bit-identical to the
    single-GPU matmul)."""
    import ctypes as C

    import torch

    from . import _lib

    L = _lib.lib()
    x = x.contiguous()
    m = x.shape[0]
    s = stream if stream is not None else torch.cuda.current_stream(x.device)
    need = L.zq_matmul_sharded_workspace_bytes(weight_shard.handle, m, n_cols, comm.world)
    with torch.cuda.stream(s):
        ws = torch.empty(need + 256, dtype=torch.uint8, device=x.device)
        y = out if out is not None else torch.empty((m, n_cols), dtype=torch.float32, device=x.device)
    ws_ptr = (ws.data_ptr() + 255) & ~255
    _lib.check(L.zq_matmul_sharded(weight_shard.handle, C.c_void_p(x.data_ptr()), m,
                                   None if bias_shard is None else C.c_void_p(bias_shard.data_ptr()),
                                   C.c_void_p(y.data_ptr()), n_cols, comm.handle, C.c_void_p(ws_ptr), need,
                                   C.c_void_p(s.cuda_stream)))
    return y
