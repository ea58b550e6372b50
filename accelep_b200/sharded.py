"""C5: the int8-weight product N-sharded across the ranks of a process group.

Y[M, N] = X[M, K] @ dequant(W[K, N]) with W int8 [K, N] and per-column fp32
scales. Rank r of W ranks holds the column block W[:, r*Nr:(r+1)*Nr] (Nr = N /
W) and its scales, computes its block of Y on its own GPU with
accel_b200_matmul_q8, and an all-gather over the group (NCCL over NVLink on
GPUs) assembles Y on every rank. There is no reduction: each output column is
computed by exactly one rank, so Y is bit-identical to the unsharded
product's columns computed by the same kernel.

Two ways to assemble Y:
  * mode "nccl": the local block goes to a buffer and NCCL's all-gather
    (all_gather_into_tensor) collects the blocks; a transpose copy makes Y.
  * mode "fused": Y lives in symmetric memory (every rank's Y mapped into every
    process); the product kernel itself stores each output element of its
    block into every rank's Y (accel_b200_matmul_q8_peers, peer stores over
    NVLink from the epilogue), then the ranks meet at a barrier over peer
    memory (accel_b200_peer_barrier, bounded wait). No copy, no separate
    collective; two Y buffers alternate so that a rank one call ahead never
    overwrites a Y a peer may still read (so a captured CUDA graph must hold
    an even number of calls).

The local product is a parameter so that the nccl gather logic can run on CPU
ranks (gloo) with a CPU product in tests.

Failure detection (mode "nccl"): with a `deadline` (seconds), the host waits
for the all-gather at most that long. A peer that died, left the group or
stalls before the collective then ends the call with CollectiveFailed after
at most the deadline, and the layer aborts the group's communicator
(torch.distributed's abort, ncclCommAbort under NCCL) so that no rank keeps
an operation in flight on it. The call is then synchronous on the host
(not for CUDA-graph capture); without a deadline the gather is queued on the
stream as usual and the process group's own timeout is the bound. The
reference surfaces such failures as the exception RunKernel turns into
ORT_EP_FAIL (src/ep.cc:1924-1934): CollectiveFailed is a RuntimeError.
"""

import ctypes
import threading
import time

import torch
import torch.distributed as dist


def shard_columns(w, scale, rank, world):
    """Column block `rank` of W [K, N] and of its scales (N % world == 0)."""
    n = w.shape[1]
    if n % world != 0:
        raise ValueError(f"N = {n} does not split into {world} equal column blocks")
    nr = n // world
    return w[:, rank * nr:(rank + 1) * nr].contiguous(), scale[rank * nr:(rank + 1) * nr].contiguous()


def _gpu_product(x, w, scale, out):
    from . import kernels as K

    return K.matmul_q8(x, w, scale, out=out)


class CollectiveFailed(RuntimeError):
    """The all-gather did not complete within the layer's deadline (a peer
    died, left or stalled); the group's communicator has been aborted."""


class ShardedQ8Linear:
    """One rank's part of the N-sharded product.

    w_shard / scale_shard: this rank's column block (shard_columns). product:
    (x, w, scale, out) -> out, the local product (default: the CUDA kernels).
    deadline: seconds the host waits for the all-gather (mode "nccl"), or
    None to queue it on the stream without a host wait.
    """

    def __init__(self, w_shard, scale_shard, group=None, product=None, mode="nccl", deadline=None):
        if mode not in ("nccl", "fused"):
            raise ValueError("mode is 'nccl' or 'fused'")
        if deadline is not None and (mode != "nccl" or deadline <= 0):
            raise ValueError("a deadline needs mode 'nccl' and a positive number of seconds")
        self.mode = mode
        self.deadline = deadline
        self.aborted = False
        self.group = group
        initialized = dist.is_available() and dist.is_initialized()
        self.world = dist.get_world_size(group) if initialized else 1
        self.rank = dist.get_rank(group) if initialized else 0
        self.w = w_shard
        self.scale = scale_shard
        self.nr = w_shard.shape[1]
        self.product = product or _gpu_product
        self._bufs = {}
        self._fused = {}
        self.status = None

    def _buffers(self, m, device):
        key = (m, str(device))
        if key not in self._bufs:
            local = torch.empty(m, self.nr, dtype=torch.float32, device=device)
            gathered = torch.empty(self.world * m, self.nr, dtype=torch.float32, device=device)
            self._bufs[key] = (local, gathered)
        return self._bufs[key]

    def _fused_state(self, m, device):
        key = (m, str(device))
        if key in self._fused:
            return self._fused[key]
        import torch.distributed._symmetric_memory as symm_mem

        group = self.group if self.group is not None else dist.group.WORLD
        n = self.world * self.nr
        ys = []
        for _ in range(2):
            y = symm_mem.empty(m, n, dtype=torch.float32, device=device)
            hdl = symm_mem.rendezvous(y, group)
            # This rank's column block in every peer's Y.
            peers = [hdl.buffer_ptrs[p] + self.rank * self.nr * 4 for p in range(self.world) if p != self.rank]
            ys.append((y, hdl, (ctypes.c_void_p * 7)(*peers), len(peers)))
        flags = symm_mem.empty(8, dtype=torch.int32, device=device)
        flags.zero_()
        fh = symm_mem.rendezvous(flags, group)
        torch.cuda.synchronize(device)
        dist.barrier(group=group)  # every rank's flags are zero before any signal
        flag_ptrs = (ctypes.c_void_p * 8)(*[fh.buffer_ptrs[p] for p in range(self.world)])
        if self.status is None:
            self.status = torch.zeros(1, dtype=torch.int32, device=device)
        epoch = torch.zeros(1, dtype=torch.int32, device=device)
        state = {"ys": ys, "next": 0, "flags": flags, "fh": fh, "flag_ptrs": flag_ptrs, "epoch": epoch}
        self._fused[key] = state
        return state

    def _forward_fused(self, x):
        from . import kernels as K
        from ._lib import Q8Plane, check, load

        lib = load()
        m, k = x.shape
        st = self._fused_state(m, x.device)
        y, _hdl, peers, n_peers = st["ys"][st["next"]]
        st["next"] ^= 1
        n = self.world * self.nr
        plane = Q8Plane(self.w.data_ptr(), self.scale.data_ptr(), 0, 0, 1)
        need = lib.accel_b200_matmul_q8_workspace(m, k, self.nr)
        ws = K._workspace(x.device, need)
        stream = K._s()
        local = y.data_ptr() + self.rank * self.nr * 4
        check(lib.accel_b200_matmul_q8_peers(ctypes.c_void_p(x.data_ptr()), x.stride(0), ctypes.byref(plane),
                                             ctypes.c_void_p(local), n, m, k, self.nr, peers, n_peers, None,
                                             K._p(ws), 0 if ws is None else ws.numel(), stream))
        check(lib.accel_b200_peer_barrier(st["flag_ptrs"], ctypes.c_void_p(st["flags"].data_ptr()), self.rank,
                                          self.world, K._p(st["epoch"]), 0, K._p(self.status), stream))
        return y

    def forward(self, x):
        """Y [M, N] on every rank."""
        if self.mode == "fused" and self.world > 1:
            return self._forward_fused(x)
        m = x.shape[0]
        local, gathered = self._buffers(m, x.device)
        self.product(x, self.w, self.scale, local)
        if self.world == 1:
            return local.clone()
        if self.deadline is None:
            dist.all_gather_into_tensor(gathered, local, group=self.group)
        else:
            self._gather_within_deadline(gathered, local)
        # [world * M, Nr] (rank-major) -> [M, world * Nr]: rank r's block is
        # columns r*Nr .. (r+1)*Nr - 1.
        return gathered.view(self.world, m, self.nr).permute(1, 0, 2).reshape(m, self.world * self.nr)

    def _gather_within_deadline(self, gathered, local):
        if self.aborted:
            raise CollectiveFailed("the communicator of this layer's group was aborted by an earlier failure")
        # The host polls the collective's completion against a monotonic
        # deadline (every backend's Work answers is_completed; not every one
        # honours a timeout in wait), spinning for the first millisecond and
        # then polling every 200 us.
        start = time.monotonic()
        end = start + self.deadline
        try:
            work = dist.all_gather_into_tensor(gathered, local, group=self.group, async_op=True)
            while not work.is_completed():
                now = time.monotonic()
                if now > end:
                    raise TimeoutError(f"not complete after {now - start:.3f} s")
                if now - start > 1e-3:
                    time.sleep(2e-4)
            work.wait()  # orders the caller's stream after the collective
        except Exception as ex:  # the deadline, or the backend's lost-peer error
            self._abort()
            raise CollectiveFailed(f"all-gather over {self.world} ranks did not complete within {self.deadline} s "
                                   f"({type(ex).__name__}: {ex}); the communicator was aborted") from ex

    def _abort(self):
        """Aborts the group's communicator (ncclCommAbort under NCCL): no
        operation stays in flight on it and later collectives on it fail. The
        abort runs on a helper thread that the caller waits for at most one
        second (a backend may hold its abort until the stalled operation
        ends); the layer refuses further calls either way."""
        self.aborted = True

        def abort():
            try:
                dist.distributed_c10d._abort_process_group(self.group)
            except Exception:  # a backend without abort: the group is left to its own timeout
                pass

        helper = threading.Thread(target=abort, name="accel-b200-abort", daemon=True)
        helper.start()
        helper.join(timeout=1.0)

    __call__ = forward
