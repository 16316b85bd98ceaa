"""Tensor-parallel reduction over NVLink peer memory for a group of ranks,
one GPU each (the host side of nd_comm_* / nd_allreduce_add_layernorm).

Every rank allocates one region in the library, the 64-byte IPC handles are
exchanged through the torch.distributed group, and each rank maps the other
ranks' regions.  A caller writes its partial sum into `partial(rows)` (a view
of its own region's current slot, e.g. as a GEMM's output) and then calls
`add_layernorm`, which sums all ranks' partials over NVLink, adds the
residual and bias and applies the LayerNorm; or it calls
`linear_add_layernorm`, which also computes the partial (the row-parallel
projection) in the same launch.  Slots alternate automatically.  All ranks
must make the same calls in the same order.
"""
import torch
import torch.distributed as dist

from . import ops


class _DeviceArray:
    """A raw device pointer seen as an array (the CUDA array interface)."""

    def __init__(self, ptr, shape, typestr):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (ptr, False), "version": 3, "strides": None}


class PeerReduce:
    def __init__(self, rows_max, d, group=None, device=None):
        self.group = group
        self.tp = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.rows_max, self.d = rows_max, d
        self.device = torch.device(device or "cuda")
        self.nbytes = ops.comm_region_bytes(rows_max, d)
        self.region, handle = ops.comm_alloc(self.nbytes)
        handles = [None] * self.tp
        dist.all_gather_object(handles, handle, group=group)
        self.regions = [self.region if r == self.rank else ops.comm_open(handles[r])
                        for r in range(self.tp)]
        self.slots = []
        for k in range(2):
            ptr = self.region + ops.comm_slot_offset(k, rows_max, d)
            t = torch.as_tensor(_DeviceArray(ptr, (rows_max, d), "<i2"), device=self.device)
            self.slots.append(t.view(torch.bfloat16))
        self.k = 0

    def partial(self, rows):
        """Where this rank writes its partial sum [rows][d] for the next call."""
        return self.slots[self.k][:rows]

    def add_layernorm(self, x, bias, gamma, beta, eps, s_out, out):
        ops.allreduce_add_layernorm(self.regions, self.rank, self.nbytes, self.rows_max, self.k,
                                    x, bias, gamma, beta, s_out, out, eps)
        self.k ^= 1
        return s_out, out

    def fused_supported(self, rows, K):
        """Whether linear_add_layernorm takes rows x K projection inputs
        (tp 1, 2, 4 or 8; rows <= 32; d a multiple of 8 up to 1024; K a
        multiple of 32)."""
        return (self.tp in (1, 2, 4, 8) and 1 <= rows <= min(32, self.rows_max)
                and self.d % 8 == 0 and 8 <= self.d <= 1024 and K >= 32 and K % 32 == 0)

    def linear_add_layernorm(self, a, w, x, bias, gamma, beta, eps, s_out, out):
        """s_out = x + Σ_r bf16(a_r · w_rᵀ) + bias, out = LayerNorm(s_out), where
        a [rows][K] and w [d][K] are this rank's shards (one launch)."""
        ops.gemm_allreduce_add_layernorm(a, w, self.regions, self.rank, self.nbytes, self.rows_max,
                                         self.k, x, bias, gamma, beta, s_out, out, eps)
        self.k ^= 1
        return s_out, out

    def close(self):
        """Unmap the peers' regions and free this rank's once no rank reads or
        maps it any more (collective: every rank calls it)."""
        if self.region is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)      # no rank reads any region any more
        for r, p in enumerate(self.regions):
            if r != self.rank:
                ops.comm_close(p)
        dist.barrier(group=self.group)      # every mapping of this region is closed
        self.slots = []
        ops.comm_free(self.region)
        self.region = None
