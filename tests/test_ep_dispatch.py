"""Expert-parallel prefill exchange (mtp_b200.ep): the dispatch plan, and the
dispatch -> local experts -> combine round trip on 2 and 4 gloo ranks (CPU)
and 2 NCCL ranks (GPU), against the layer over all experts on one device."""
import multiprocessing as mp
import socket

import pytest
import torch

import ep_workers
from mtp_b200.ep import plan_dispatch

REL_L2 = 1e-2
NORM_MAX_ABS = 2e-2


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(target, world: int, cfg: dict, timeout: float = 300.0):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=target, args=(r, world, port, cfg, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            rank, res, err = q.get(timeout=timeout)
            results[rank] = (res, err)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    return results


def test_plan_dispatch_dedups_rows_and_marks_foreign_pairs():
    # E = 8 over 2 ranks: experts 0-3 on rank 0, 4-7 on rank 1; id -1 is never sent
    ids = torch.tensor([[0, 5], [1, 2], [7, 6], [3, -1]], dtype=torch.int32)
    w = torch.tensor([[0.6, 0.4], [0.5, 0.5], [0.7, 0.3], [1.0, 0.0]])
    p = plan_dispatch(ids, w, 8, 2)
    assert p.counts == [3, 2]
    assert p.tokens.tolist() == [0, 1, 3, 0, 2]
    assert p.local_ids.tolist() == [[0, -1], [1, 2], [3, -1], [-1, 1], [3, 2]]
    assert torch.equal(p.local_weights, torch.tensor([[0.6, 0.0], [0.5, 0.5], [1.0, 0.0], [0.0, 0.4], [0.7, 0.3]]))
    # every valid pair is sent exactly once, to its owner
    assert int((p.local_ids >= 0).sum()) == int((ids >= 0).sum())


def test_plan_dispatch_rejects_uneven_shards():
    with pytest.raises(ValueError):
        plan_dispatch(torch.zeros((2, 2), dtype=torch.int32), torch.zeros((2, 2)), 6, 4)


@pytest.mark.parametrize("world,cfg", [
    (2, dict(E=8, H=256, I=128, k=2, G=128, shared=True, M=[6, 5])),
    (4, dict(E=16, H=256, I=128, k=4, G=64, shared=False, M=[5, 0, 7, 3])),
    (2, dict(E=8, H=256, I=128, k=2, G=128, shared=True, M=[4, 4], skip_rank=1)),
    # the all-gather / reduce-scatter form (equal tokens per rank)
    (2, dict(E=8, H=256, I=128, k=2, G=128, shared=True, M=[5, 5], gather=True)),
    (4, dict(E=16, H=256, I=128, k=4, G=64, shared=False, M=[3, 3, 3, 3], gather=True)),
    (2, dict(E=8, H=256, I=128, k=2, G=128, shared=True, M=[4, 4], skip_rank=0, gather=True)),
])
def test_ep_round_trip_on_gloo_ranks_matches_single_device(world, cfg):
    res = _run(ep_workers.cpu_rank, world, cfg)
    assert sorted(res) == list(range(world))
    for rank, (r, err) in res.items():
        assert err is None, f"rank {rank}: {err}"
        assert r[0] <= REL_L2 and r[1] <= NORM_MAX_ABS, f"rank {rank}: rel-L2 {r[0]}, max-abs {r[1]}"


@pytest.mark.gpu
@pytest.mark.parametrize("gather", [False, True])
def test_ep_round_trip_on_two_gpus_matches_single_gpu_layer(gather):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    cfg = dict(E=256, H=2048, I=512, k=8, G=128, M=512, gather=gather)
    res = _run(ep_workers.gpu_rank, 2, cfg, timeout=600.0)
    for rank, (r, err) in res.items():
        assert err is None, f"rank {rank}: {err}"
        assert r[0] <= REL_L2 and r[1] <= NORM_MAX_ABS, f"rank {rank}: rel-L2 {r[0]}, max-abs {r[1]}"
