"""Output-row sharding of mul_mat across ranks (one process per GPU).

Every output of mul_mat is an independent chain of LNS additions, so
splitting the M output rows into contiguous blocks changes no bit: rank r
keeps the k-major weight columns [m0, m1) of every slice (its own [K][M_r]
matrix), computes dst[:, m0:m1] and the ranks exchange their blocks with one
all-gather.  Monte chains start from their global output index, so the Monte
result is shard-invariant too (the C ABI takes the global row offset through
the weight pointer only; callers that shard Monte mul_mats pass each rank's
start state, see monte_seed_for_shard).

The all-gather yields [world][N][M_r]; dst in ggml order is [N][M], i.e. the
gathered blocks permuted (gather_layout).
"""


def row_range(M, world, rank):
    """[m0, m1) of rank's rows: contiguous blocks, the first M % world ranks one row longer."""
    base, extra = divmod(M, world)
    m0 = rank * base + min(rank, extra)
    return m0, m0 + base + (1 if rank < extra else 0)


def equal_shards(M, world):
    return M % world == 0


def shard_weights_kmajor(w_kmajor, M, world, rank):
    """The rank's columns of a k-major [K][M] weight (a torch tensor or numpy array)."""
    m0, m1 = row_range(M, world, rank)
    return w_kmajor.reshape(-1, M)[:, m0:m1]


def gather_layout(gathered, world, N, Mr):
    """[world][N][Mr] -> [N][world*Mr] (ggml dst order) for equal shards."""
    return gathered.reshape(world, N, Mr).permute(1, 0, 2).reshape(N, world * Mr)


def all_gather_rows(dst_shard, world, group=None):
    """All-gathers equal [N][Mr] row blocks into the full [N][world*Mr] output
    (NCCL: one all_gather_into_tensor; gloo, for CPU tests: all_gather).  The
    codes travel as raw bytes: neither backend has a 16-bit integer type, and
    a gather does no arithmetic."""
    import torch
    import torch.distributed as dist
    N, Mr = dst_shard.shape
    src = dst_shard.contiguous().view(-1).view(torch.uint8)
    if dist.get_backend(group) == "nccl":
        out = torch.empty(world * src.numel(), dtype=torch.uint8, device=dst_shard.device)
        dist.all_gather_into_tensor(out, src, group=group)
    else:
        parts = [torch.empty_like(src) for _ in range(world)]
        dist.all_gather(parts, src, group=group)
        out = torch.cat(parts)
    return gather_layout(out.view(dst_shard.dtype), world, N, Mr)


def monte_seed_for_shard(seed, jump, M, N, K, rank, world, slices=1):
    """LFSR state where rank's first chain starts, given the op's seed, for a
    single-slice mul_mat: the chain of global output o = m * N + n starts
    o * (K-1) draws after the op's seed, so the rank's outputs are the global
    ones shifted by m0 * N.  jump(s, n) is the LFSR jump-ahead.

    With several slices (z > 0) the kernels number chain (z, m, n) as
    (z * M_local + m) * N + n, so a shard's chains are not one contiguous run
    of the global order and no single start state reproduces it: refused."""
    if slices != 1:
        raise ValueError("monte_seed_for_shard: a sharded Monte mul_mat must have a single slice (got %d)" % slices)
    m0, _ = row_range(M, world, rank)
    return jump(seed, m0 * N * max(K - 1, 0))


# ---------------------------------------------------------------------------
# Failure detection on the host.  A rank that never joins, or leaves between
# steps, is noticed by the others on the host -- through the rendezvous store,
# with a deadline -- before their next launch, so no kernel or collective is
# left waiting on it.  (The device-side waits have their own bounds: the peer
# barrier of the fused gather gives up after a fixed number of polls and
# reports a status.)
# ---------------------------------------------------------------------------

class ShardError(RuntimeError):
    """A rank did not join, or is gone; .ranks names the missing ones."""

    def __init__(self, msg, ranks=()):
        super().__init__(msg)
        self.ranks = tuple(ranks)


def init_group(backend, rank, world, port, addr="127.0.0.1", timeout_s=30.0):
    """init_process_group over a TCPStore that rank 0 hosts, with a deadline:
    if any rank does not join within timeout_s, every rank that did raises
    ShardError (rank 0 after waiting for the workers, the others after failing
    to reach rank 0's store).  Returns the store (for StepGuard).  The process
    group's own timeout is timeout_s as well, so a collective that a vanished
    peer never joins ends with an error instead of hanging."""
    import datetime
    import torch.distributed as dist
    td = datetime.timedelta(seconds=timeout_s)
    try:
        store = dist.TCPStore(addr, port, world, rank == 0, timeout=td, wait_for_workers=True)
        store.set("lnsb/joined/%d" % rank, "1")
        store.wait(["lnsb/joined/%d" % r for r in range(world)], td)
    except Exception as e:                                   # torch raises DistStoreError / RuntimeError
        raise ShardError("rank %d: the group of %d did not assemble within %.1f s (%s)"
                         % (rank, world, timeout_s, type(e).__name__)) from e
    dist.init_process_group(backend, store=store, rank=rank, world_size=world, timeout=td)
    return store


class StepGuard:
    """Per-step heartbeat through the store.  enter(step) is called before a
    step's first launch: it records this rank's arrival and waits, at most
    timeout_s, for every other rank's; a rank that announced leave() (or never
    arrives) makes enter raise ShardError naming it, on every rank still
    present, before any of them launches the step's kernels or collectives."""

    def __init__(self, store, rank, world, timeout_s=10.0, poll_s=0.01):
        self.store, self.rank, self.world = store, rank, world
        self.timeout_s, self.poll_s = timeout_s, poll_s

    def _key(self, step, r):
        return "lnsb/step/%d/%d" % (step, r)

    def _left(self):
        return [r for r in range(self.world) if r != self.rank and self.store.check(["lnsb/left/%d" % r])]

    def enter(self, step):
        import time
        self.store.set(self._key(step, self.rank), "1")
        deadline = time.monotonic() + self.timeout_s
        while True:
            left = self._left()
            if left:
                raise ShardError("step %d: rank(s) %s left the group" % (step, left), left)
            missing = [r for r in range(self.world) if not self.store.check([self._key(step, r)])]
            if not missing:
                return
            if time.monotonic() >= deadline:
                raise ShardError("step %d: rank(s) %s did not arrive within %.1f s" % (step, missing, self.timeout_s),
                                 missing)
            time.sleep(self.poll_s)

    def leave(self):
        """This rank leaves between steps (none of its work in flight)."""
        self.store.set("lnsb/left/%d" % self.rank, "1")
