"""Host logic of the split-KV path, on CPU: the range partition and the
all-gather + log-sum-exp exchange between world-size-2 gloo ranks, with the
oracle computing each rank's partial and the merge."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import load_package  # spawned ranks import this module without pytest

load_package()
import nyion_rs_b200.splitkv as S  # noqa: E402
import oracle as O  # noqa: E402

N_KV, D, PT, H = 4, 64, 16, 32


def test_rank_range_partition():
    for total in [1, 63, 64, 1000, 1048576, 1048577]:
        for world in [1, 2, 3, 4, 8]:
            rs = [S.rank_range(r, world, total) for r in range(world)]
            assert rs[0][0] == 0 and rs[-1][1] == total
            for (a, b), (c, d) in zip(rs, rs[1:]):
                assert b == c and a <= b
            for a, _ in rs[1:]:
                assert a % S.CHUNK == 0 or a == total
            sizes = [b - a for a, b in rs]
            assert max(sizes) - min(sizes) <= S.CHUNK
    with pytest.raises(ValueError):
        S.rank_range(2, 2, 100)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _case(seed=5, T=900):
    rng = np.random.default_rng(seed)
    src = rng.standard_normal((T, N_KV, 2, D), dtype=np.float32)
    q4 = O.q4_quantize_rows(src, D)
    pages = (T + PT - 1) // PT
    pool = np.zeros((pages, N_KV, 2, PT, 40), np.uint8)
    for t in range(T):
        pool[t // PT, :, :, t % PT] = q4[t]
    table = np.arange(pages, dtype=np.int32)[None]
    q = rng.standard_normal((1, H, D), dtype=np.float32)
    return q, pool, table, T


def _worker(rank, world, port, result_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q, pool, table, T = _case()
        lo, hi = S.rank_range(rank, world, T)
        part = torch.from_numpy(O.decode_q4_partial(q, pool, table, lo, hi, N_KV, D, PT))
        parts = S.exchange(part)
        assert parts.shape == (world, 1, H, D + 2)
        out = O.lse_combine(parts.numpy())
        np.save(result_path + f".{rank}.npy", out)
    finally:
        dist.destroy_process_group()


def test_gloo_exchange_matches_single_rank(tmp_path):
    world = 2
    path = str(tmp_path / "out")
    mp.start_processes(_worker, args=(world, _free_port(), path), nprocs=world, join=True,
                       start_method="spawn")
    q, pool, table, T = _case()
    whole = O.lse_combine(O.decode_q4_partial(q, pool, table, 0, T, N_KV, D, PT)[None])
    for r in range(world):
        got = np.load(path + f".{r}.npy")
        assert np.abs(got - whole).max() < 1e-5
