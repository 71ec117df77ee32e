"""Process meshes over torch.distributed: the mesh shapes of the reference's
``create_simple_mesh`` / ``_get_batch_axis`` (``sharding/sharding_utils.py:21-179``).

One process per GPU; ranks are laid out row-major over the mesh axes, so the last
axis is the fastest-varying (consecutive ranks, i.e. GPUs of one node on NVLink).

* ``("data",)``           -- pure data parallelism (default);
* ``("nodes", "gpus")``   -- hierarchical data parallelism (``hierarchical=True``): an
  intra-node group per node and a cross-node group per local rank, for two-level
  gradient reduction; on one node (``allow_single_node_hierarchical``) it is (1, N);
* ``("dp", "tp")``        -- tensor parallelism over consecutive ranks (``tp_size``), data
  parallelism across the TP groups;
* ``("tp",)``             -- pure tensor parallelism (``tp_size`` = world size).

``Mesh.group(axis)`` is the process group of this rank along an axis (every rank
creates every group, in the same order, as ``new_group`` requires);
``Mesh.batch_axis`` names the axes the batch is split over (``None``: replicated);
``Mesh.batch_rank`` / ``batch_world`` give this rank's data shard.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, Optional, Tuple, Union

import numpy as np
import torch.distributed as dist


@dataclass
class Mesh:
    axis_names: Tuple[str, ...]
    shape: Tuple[int, ...]
    rank: int
    groups: Dict[str, object] = field(default_factory=dict)

    @property
    def coords(self) -> Tuple[int, ...]:
        return tuple(int(c) for c in np.unravel_index(self.rank, self.shape))

    def size(self, axis: str) -> int:
        return self.shape[self.axis_names.index(axis)]

    def coord(self, axis: str) -> int:
        return self.coords[self.axis_names.index(axis)]

    def group(self, axis: str):
        return self.groups[axis]

    @property
    def batch_axis(self) -> Optional[Union[str, Tuple[str, ...]]]:
        names = self.axis_names
        if "tp" in names:
            return "dp" if "dp" in names else None
        if names == ("nodes", "gpus"):
            return ("nodes", "gpus")
        return names[0]

    @property
    def batch_world(self) -> int:
        ax = self.batch_axis
        if ax is None:
            return 1
        axes = (ax,) if isinstance(ax, str) else ax
        return int(np.prod([self.size(a) for a in axes]))

    @property
    def batch_rank(self) -> int:
        ax = self.batch_axis
        if ax is None:
            return 0
        axes = (ax,) if isinstance(ax, str) else ax
        r = 0
        for a in axes:
            r = r * self.size(a) + self.coord(a)
        return r


def mesh_shape(world: int, hierarchical: bool = False, tp_size: int = 1, gpus_per_node: Optional[int] = None,
               allow_single_node_hierarchical: bool = False,
               per_gpu_processes: bool = False) -> Tuple[Tuple[str, ...], Tuple[int, ...]]:
    """(axis names, shape) for ``world`` ranks, without creating groups.

    ``per_gpu_processes``: every GPU is its own process (torchrun), which is the
    reference's multi-process branch, where a (dp, tp) mesh is allowed on one node; its
    single-process branch (one process driving all local GPUs) requires tp = all GPUs."""
    gpn = gpus_per_node or world
    if world % gpn:
        raise ValueError(f"world size {world} is not a multiple of gpus_per_node {gpn}")
    nodes = world // gpn
    if tp_size > 1:
        if world % tp_size:
            raise ValueError(f"world size {world} must be divisible by tp_size {tp_size}")
        if nodes == 1 and tp_size != world and not per_gpu_processes:
            raise ValueError(f"on one node tp_size ({tp_size}) must equal the number of GPUs ({world})")
        dp = world // tp_size
        return (("tp",), (tp_size,)) if dp == 1 else (("dp", "tp"), (dp, tp_size))
    if hierarchical and (nodes > 1 or allow_single_node_hierarchical):
        return ("nodes", "gpus"), (nodes, gpn)
    return ("data",), (world,)


def create_mesh(hierarchical: bool = False, tp_size: int = 1, gpus_per_node: Optional[int] = None,
                allow_single_node_hierarchical: bool = False, per_gpu_processes: bool = False) -> Mesh:
    """Build the mesh of the current process group and its per-axis groups."""
    world, rank = dist.get_world_size(), dist.get_rank()
    names, shape = mesh_shape(world, hierarchical, tp_size, gpus_per_node, allow_single_node_hierarchical,
                              per_gpu_processes)
    ranks = np.arange(world).reshape(shape)
    m = Mesh(names, shape, rank)
    for ax, name in enumerate(names):
        moved = np.moveaxis(ranks, ax, -1).reshape(-1, shape[ax])    # every line along this axis
        for line in moved:
            g = dist.new_group([int(r) for r in line]) if len(names) > 1 else dist.group.WORLD
            if rank in line:
                m.groups[name] = g
    return m
