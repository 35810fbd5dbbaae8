"""Two-dimensional process layouts: tensor parallelism inside groups of consecutive ranks (one
NVSwitch domain's GPUs), data parallelism across the groups.

    mesh = Mesh(comm, tp=4)              # world = tp * dp; rank = dp_index * tp + tp_index
    mlp = TensorParallelMLP(mesh.tp, hidden, ffn)
    dp = DataParallelSync(mesh.dp, grads)

Built on ``Communicator.split`` (collective over ``comm``). The reference has no parallelism
layer; its communicator's machine view (OriginCCL include/communicator.h:19-75) is the closest
notion of a process grid.
"""
from __future__ import annotations

class Mesh:
    """``tp`` / ``dp``: this rank's tensor-parallel and data-parallel communicators."""

    def __init__(self, comm, tp: int) -> None:
        world = comm.world_size
        if tp < 1 or world % tp != 0:
            raise ValueError(f"tp={tp} must divide the world size {world}")
        self.comm = comm
        self.tp_size = tp
        r = comm.rank
        self.tp = comm.split(r // tp, key=r % tp)   # consecutive ranks
        self.dp = comm.split(r % tp, key=r // tp)   # the same position in every TP group

    @property
    def dp_size(self) -> int:
        return self.comm.world_size // self.tp_size

    def destroy(self) -> None:
        for c in (self.tp, self.dp):
            if c is not None:
                c.destroy()
        self.tp = self.dp = None
