"""Process meshes on 4 gloo ranks: shapes, per-axis groups and batch-axis resolution."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from sigma0_b200.parallel.mesh import mesh_shape


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_mesh_shapes():
    assert mesh_shape(8) == (("data",), (8,))
    assert mesh_shape(8, hierarchical=True, gpus_per_node=4) == (("nodes", "gpus"), (2, 4))
    assert mesh_shape(4, hierarchical=True) == (("data",), (4,))
    assert mesh_shape(4, hierarchical=True, allow_single_node_hierarchical=True) == (("nodes", "gpus"), (1, 4))
    assert mesh_shape(16, tp_size=4, gpus_per_node=4) == (("dp", "tp"), (4, 4))
    assert mesh_shape(8, tp_size=8) == (("tp",), (8,))
    assert mesh_shape(16, tp_size=8, gpus_per_node=4) == (("dp", "tp"), (2, 8))     # TP across two nodes
    with pytest.raises(ValueError):
        mesh_shape(8, tp_size=4)                                                    # one node: tp must be 8
    with pytest.raises(ValueError):
        mesh_shape(8, tp_size=3, gpus_per_node=4)


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from sigma0_b200.parallel.mesh import create_mesh
    res = {}
    for name, kw in [("data", {}), ("hier", dict(hierarchical=True, gpus_per_node=2)),
                     ("dptp", dict(tp_size=2, gpus_per_node=2)), ("tp", dict(tp_size=4))]:
        m = create_mesh(**kw)
        sums = {}
        for ax in m.axis_names:
            t = torch.tensor([float(rank)])
            dist.all_reduce(t, group=m.group(ax))
            sums[ax] = float(t)
        res[name] = (m.axis_names, m.shape, m.coords, sums, m.batch_axis, m.batch_rank, m.batch_world)
    q.put((rank, res))
    dist.barrier()
    dist.destroy_process_group()


def test_mesh_groups_on_gloo():
    world, port = 4, _port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    out = dict(q.get(timeout=120) for _ in range(world))
    for p in ps:
        p.join(60)
    for r in range(world):
        d = out[r]["data"]
        assert d[0] == ("data",) and d[3]["data"] == 6.0 and d[4] == "data" and d[5] == r
        h = out[r]["hier"]
        assert h[1] == (2, 2) and h[2] == divmod(r, 2)
        assert h[3]["gpus"] == (0 + 1 if r < 2 else 2 + 3) and h[3]["nodes"] == (0 + 2 if r % 2 == 0 else 1 + 3)
        assert h[4] == ("nodes", "gpus") and h[5] == r and h[6] == 4
        t = out[r]["dptp"]
        assert t[0] == ("dp", "tp") and t[3]["tp"] == (1.0 if r < 2 else 5.0)
        assert t[4] == "dp" and t[5] == r // 2 and t[6] == 2
        p = out[r]["tp"]
        assert p[0] == ("tp",) and p[4] is None and p[6] == 1
