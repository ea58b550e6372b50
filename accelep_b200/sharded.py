"""C5: the int8-weight product N-sharded across the ranks of a process group.

Y[M, N] = X[M, K] @ dequant(W[K, N]) with W int8 [K, N] and per-column fp32
scales. Rank r of W ranks holds the column block W[:, r*Nr:(r+1)*Nr] (Nr = N /
W) and its scales, computes its block of Y on its own GPU with
accel_b200_matmul_q8, and an all-gather over the group (NCCL over NVLink on
GPUs) assembles Y on every rank. There is no reduction: each output column is
computed by exactly one rank, so Y is bit-identical to the unsharded
product's columns computed by the same kernel.

The local product is a parameter so that the gather logic can run on CPU
ranks (gloo) with a CPU product in tests.
"""

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


class ShardedQ8Linear:
    """One rank's part of the N-sharded product.

    w_shard / scale_shard: this rank's column block (shard_columns). product:
    (x, w, scale, out) -> out, the local product (default: the CUDA kernels).
    """

    def __init__(self, w_shard, scale_shard, group=None, product=None):
        self.group = group
        initialized = dist.is_available() and dist.is_initialized()
        self.world = dist.get_world_size(group) if initialized else 1
        self.rank = dist.get_rank(group) if initialized else 0
        self.w = w_shard
        self.scale = scale_shard
        self.nr = w_shard.shape[1]
        self.product = product or _gpu_product
        self._bufs = {}

    def _buffers(self, m, device):
        key = (m, str(device))
        if key not in self._bufs:
            local = torch.empty(m, self.nr, dtype=torch.float32, device=device)
            gathered = torch.empty(self.world * m, self.nr, dtype=torch.float32, device=device)
            self._bufs[key] = (local, gathered)
        return self._bufs[key]

    def forward(self, x):
        """Y [M, N] on every rank."""
        m = x.shape[0]
        local, gathered = self._buffers(m, x.device)
        self.product(x, self.w, self.scale, local)
        if self.world == 1:
            return local.clone()
        dist.all_gather_into_tensor(gathered, local, group=self.group)
        # [world * M, Nr] (rank-major) -> [M, world * Nr]: rank r's block is
        # columns r*Nr .. (r+1)*Nr - 1.
        return gathered.view(self.world, m, self.nr).permute(1, 0, 2).reshape(m, self.world * self.nr)

    __call__ = forward
