"""Row sharding of the GEMM -> LayerNorm path across the GPUs of one node.

GEMM rows and LayerNorm rows are independent, so a rank computes the rows
[r0, r1) of X with the whole of W on its own device: Z = X[r0:r1] W, then
Y = LayerNorm(Z) with replicated gamma/beta. There is no exchange on the data
path; the gathered output, when a caller wants one, is a separate step.

One process drives one GPU (RANK / LOCAL_RANK / WORLD_SIZE from the launcher).
Each rank opens its own context "cuda:LOCAL_RANK" and calls the unchanged
reference entry points (pr_matmul_f32, pr_layer_norm_f32) on descriptors of its
shard; the synthetic inputs of a shard are the same draws the unsharded tensor
would use, so the union of the shards is bit-identical to one-device results.
"""
import os
from dataclasses import dataclass

from . import b200
from .native import Context
from .tensor import TensorDescriptor, layer_norm_into, matmul_into, operators_of


def row_range(rows, world, rank):
    """Balanced contiguous [r0, r1) of `rows` for `rank` of `world`."""
    if not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    base, extra = divmod(rows, world)
    r0 = rank * base + min(rank, extra)
    return r0, r0 + base + (1 if rank < extra else 0)


@dataclass(frozen=True)
class Topology:
    rank: int
    world: int
    local_rank: int

    @classmethod
    def from_environment(cls):
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        local = int(os.environ.get("LOCAL_RANK", str(rank)))
        return cls(rank, world, local)

    @property
    def selector(self):
        return f"cuda:{self.local_rank}"


class ChainShard:
    """One rank's part of Y = LayerNorm(X W) for X [rows, k], W [k, n].

    Buffers live on the rank's device for the object's lifetime: X rows
    [r0, r1), W, gamma, beta, the GEMM output Z and the result Y.
    Inputs come from the seeded stream of `seed`: X ~ N(0, 1) first, then
    W ~ N(0, w_std); gamma = 1, beta = 0 unless given.
    """

    def __init__(self, context, rows, k, n, world=1, rank=0, *, seed=4, w_std=1.0 / 64.0, epsilon=1e-5):
        self.context = context
        self.rows, self.k, self.n, self.epsilon = rows, k, n, epsilon
        self.r0, self.r1 = row_range(rows, world, rank)
        self.local_rows = self.r1 - self.r0
        self.resources = operators_of(context)
        self.queue = self.resources.queue
        m = self.local_rows
        self.x = context.buffer(4 * m * k)
        self.w = context.buffer(4 * k * n)
        self.gamma = context.buffer(4 * n)
        self.beta = context.buffer(4 * n)
        self.z = context.buffer(4 * m * n)
        self.y = context.buffer(4 * m * n)
        self.xd = TensorDescriptor(self.x, (m, k))
        self.wd = TensorDescriptor(self.w, (k, n))
        self.gd = TensorDescriptor(self.gamma, (n,))
        self.bd = TensorDescriptor(self.beta, (n,))
        self.zd = TensorDescriptor(self.z, (m, n))
        self.yd = TensorDescriptor(self.y, (m, n))
        self.seed, self.w_std = seed, w_std
        self.w_prepared = None  # b200.PreparedMatrix of W once prepare_weights() ran

    def prepare_weights(self):
        """Prepare W once (its TF32 pair and a copy, pr_b200_matmul_prepare_f32), so
        that every later step reads the prepared form instead of splitting W again.
        Results are unchanged bit for bit; a W written after this call is not seen."""
        if self.w_prepared is not None:
            self.w_prepared.close()
        self.w_prepared = b200.PreparedMatrix(self.queue, self.resources.module, self.context, self.wd,
                                              k=self.k, n=self.n)

    def _matmul(self, xd, zd, rows):
        if self.w_prepared is None:
            return matmul_into(self.queue, self.resources.module, xd, self.wd, zd, m=rows, n=self.n, k=self.k)
        return b200.matmul_prepared_into(self.queue, self.resources.module, xd, self.w_prepared.descriptor, zd,
                                         m=rows, n=self.n, k=self.k)

    def fill_synthetic(self, gamma=1.0, beta=0.0):
        """Device-side generation of this shard's inputs (draw offsets of the full stream)."""
        events = [
            b200.fill_synthetic_into(self.queue, self.xd, seed=self.seed, first_draw=2 * self.r0 * self.k,
                                     distribution=b200.NORMAL, p0=0.0, p1=1.0),
            b200.fill_synthetic_into(self.queue, self.wd, seed=self.seed, first_draw=2 * self.rows * self.k,
                                     distribution=b200.NORMAL, p0=0.0, p1=self.w_std),
        ]
        import numpy as np
        self.gamma.write(np.full(self.n, gamma, np.float32))
        self.beta.write(np.full(self.n, beta, np.float32))
        for e in events:
            if e is not None:
                e.wait()
                e.close()

    def step(self, gathered=None):
        """Enqueue Z = X W and Y = LayerNorm(Z); with `gathered` (a GatheredOutput)
        the LayerNorm also writes its rows into every rank's gathered Y. Returns the
        two events."""
        mm = self._matmul(self.xd, self.zd, self.local_rows)
        if gathered is None:
            ln = layer_norm_into(self.queue, self.resources.module, self.zd, self.gd, self.bd, self.yd,
                                 epsilon=self.epsilon)
        else:
            ln = b200.layer_norm_gather_into(self.queue, self.resources.module, self.zd, self.gd, self.bd,
                                             self.yd, gathered.targets, row_offset=self.r0, epsilon=self.epsilon)
        return mm, ln

    def step_from_host(self, x_host, y_host, slices=8, gathered=None):
        """One step with the input X and the output Y in host memory, pipelined.

        x_host / y_host are addresses of this shard's [local_rows, k] and
        [local_rows, n] float32 host arrays (page-locked, or the copies do not
        overlap). The rows are cut into `slices` slices (multiples of 128 rows, the
        GEMM tile height); per slice the queue gets an upload of the X rows, Z = X W,
        Y = LayerNorm(Z) and a download of the Y rows, all enqueued at once. The
        copies are stream-ordered (pr_b200_buffer_write_async / read_async), so the
        upload of slice i+1 and the download of slice i-1 run on the copy engines
        while slice i computes. Returns the events in submission order; the host
        arrays must stay valid until the last one completes.
        """
        m, k, n = self.local_rows, self.k, self.n
        tile = 128
        cuts = sorted({min(m, -(-m * i // slices) // tile * tile) for i in range(1, slices)} | {0, m})
        events = []
        for lo, hi in zip(cuts, cuts[1:]):
            rows = hi - lo
            xo, yo = 4 * lo * k, 4 * lo * n
            events.append(b200.write_async(self.queue, self.x, x_host + xo, offset=xo, nbytes=4 * rows * k))
            zd = TensorDescriptor(self.z, (rows, n), yo)
            yd = TensorDescriptor(self.y, (rows, n), yo)
            events.append(self._matmul(TensorDescriptor(self.x, (rows, k), xo), zd, rows))
            if gathered is None:
                events.append(layer_norm_into(self.queue, self.resources.module, zd, self.gd, self.bd, yd,
                                              epsilon=self.epsilon))
            else:
                events.append(b200.layer_norm_gather_into(self.queue, self.resources.module, zd, self.gd, self.bd,
                                                          yd, gathered.targets, row_offset=self.r0 + lo,
                                                          epsilon=self.epsilon))
            events.append(b200.read_async(self.queue, self.y, y_host + yo, offset=yo, nbytes=4 * rows * n))
        return [e for e in events if e is not None]

    def flops(self):
        return 2 * self.local_rows * self.n * self.k

    def close(self):
        if self.w_prepared is not None:
            self.w_prepared.close()
        for buf in (self.x, self.w, self.gamma, self.beta, self.z, self.y):
            buf.close()


class GatheredOutput:
    """A [rows, columns] tensor on every rank that all ranks write their rows into.

    Each rank allocates its copy, exports it, and maps every other rank's copy
    into its own context; `exchange(value)` must return every rank's value in rank
    order (any host channel: a gloo all_gather_object, a shared dict, ...). The
    fused LayerNorm writes rows straight into all copies over NVLink.
    """

    def __init__(self, context, rows, columns, exchange, rank):
        self.local = context.buffer(4 * rows * columns)
        handles = exchange(b200.export_buffer(self.local))
        self.peers = [b200.import_buffer(context, h) for r, h in enumerate(handles) if r != rank]
        self.targets = [TensorDescriptor(buf, (rows, columns)) for buf in [self.local] + self.peers]

    def close(self):
        for buf in self.peers:
            buf.close()
        self.local.close()


def open_rank_context():
    """The calling rank's topology and its context on cuda:LOCAL_RANK."""
    topology = Topology.from_environment()
    return topology, Context(topology.selector)
