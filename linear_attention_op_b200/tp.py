"""Head-parallel tensor parallelism: the shard plan and the NCCL communicator handle.

Rank r of G owns k-heads [r*Hk/G, (r+1)*Hk/G) and v-heads [r*Hv/G, (r+1)*Hv/G).  GQA keeps v-head h with
k-head h / (Hv/Hk), so each rank's v-heads read only its own k-heads.  in_proj is split by rows of the HF
weights (= output columns): q, k and the conv taps of the rank's k-heads, v, z, a, b of its v-heads;
out_proj is split by columns of the HF weight (rows of W_o^T), giving a partial [N, hidden] that one
all-reduce sums.  The reference splits the same way across the Tensix cores of one chip
(9B/gdn_layer.py:7-19,81-115; 0.8B/gdn_l1.py:7-15,103-112) and notes that the head split extends across
chips (0.8B/OPTIMIZATION.md:252-253).  ``libgdn_b200.so`` applies this plan in gdn_layer_create; the
Python version below is the same plan, used by the CPU (gloo) tests to check the partition on the oracle.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, replace

from . import _lib

HEAD_DIM = 128


@dataclass(frozen=True)
class ShardPlan:
    rank: int
    world: int
    k_heads: tuple[int, int]  # [start, stop)
    v_heads: tuple[int, int]


def shard_plan(num_k_heads: int, num_v_heads: int, rank: int, world: int) -> ShardPlan:
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} / world {world}")
    if num_k_heads % world or num_v_heads % world:
        raise ValueError(f"world {world} must divide num_k_heads {num_k_heads} and num_v_heads {num_v_heads}")
    hk, hv = num_k_heads // world, num_v_heads // world
    return ShardPlan(rank, world, (rank * hk, (rank + 1) * hk), (rank * hv, (rank + 1) * hv))


def shard_weights(w, rank: int, world: int):
    """This rank's shard of an oracle-style weight object (fields w_qkv, w_z, ..., num_k_heads,
    num_v_heads); returns an object of the same type describing a layer with the local head counts."""
    p = shard_plan(w.num_k_heads, w.num_v_heads, rank, world)
    kd = w.num_k_heads * HEAD_DIM
    (k0, k1), (v0, v1) = p.k_heads, p.v_heads
    ks = slice(k0 * HEAD_DIM, k1 * HEAD_DIM)
    vs = slice(v0 * HEAD_DIM, v1 * HEAD_DIM)
    import torch

    rows = torch.cat([torch.arange(kd)[ks], kd + torch.arange(kd)[ks], 2 * kd + torch.arange(w.num_v_heads * HEAD_DIM)[vs]])
    return replace(
        w, w_qkv=w.w_qkv[rows], w_z=w.w_z[vs], w_a=w.w_a[v0:v1], w_b=w.w_b[v0:v1], conv_w=w.conv_w[rows],
        a_log=w.a_log[v0:v1], dt_bias=w.dt_bias[v0:v1], w_out=w.w_out[:, vs],
        num_k_heads=k1 - k0, num_v_heads=v1 - v0,
    )


class Communicator:
    """A gdn_comm* (NCCL communicator created inside libgdn_b200.so) over a group of ranks."""

    ID_BYTES = 128

    def __init__(self, unique_id: bytes, rank: int, world: int):
        handle = ctypes.c_void_p()
        buf = ctypes.create_string_buffer(bytes(unique_id), self.ID_BYTES)
        _lib.call("gdn_comm_create", buf, self.ID_BYTES, rank, world, ctypes.byref(handle))
        self.handle = handle
        self.rank, self.world = rank, world

    @classmethod
    def unique_id(cls) -> bytes:
        buf = ctypes.create_string_buffer(cls.ID_BYTES)
        _lib.call("gdn_comm_get_unique_id", buf, cls.ID_BYTES)
        return buf.raw

    @classmethod
    def from_process_group(cls, group=None) -> "Communicator":
        """Rank 0 makes the NCCL id and broadcasts it over an initialised torch.distributed group."""
        import torch.distributed as dist

        rank, world = dist.get_rank(group), dist.get_world_size(group)
        obj = [cls.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0, group=group)
        return cls(obj[0], rank, world)

    def allgather_(self, buf, stream=None):
        """In place over the group (gdn_comm_allgather): buf (contiguous, on this rank's device) is split into
        world equal parts along its bytes; part r comes from rank r."""
        import torch

        if not buf.is_contiguous() or (buf.numel() * buf.element_size()) % self.world:
            raise ValueError("allgather_ wants a contiguous buffer whose bytes divide by the world size")
        s = stream if stream is not None else torch.cuda.current_stream(buf.device)
        _lib.call("gdn_comm_allgather", self.handle, ctypes.c_void_p(buf.data_ptr()),
                  buf.numel() * buf.element_size() // self.world, ctypes.c_void_p(s.cuda_stream))
        return buf

    def close(self) -> None:
        if getattr(self, "handle", None) is not None and self.handle.value:
            _lib.lib().gdn_comm_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
