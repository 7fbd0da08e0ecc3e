"""Rank program for the multi-GPU split-KV test (launched by torchrun from
tests/test_splitkv_multi_gpu.py).  Every rank uploads only its own pages, runs
SplitKVDecoder.step in both exchange modes — "p2p" (rows written into every
rank's mailbox by the decode's merging CTAs, combined by the exchange kernel
after a bounded wait)
and "collective" (NCCL all-gather + LSE combine) — for several steps, inside
and outside a CUDA graph, and checks the merged output against the one-GPU
decode over the whole context and the oracle."""
import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
from conftest import load_package  # noqa: E402

load_package()
import nyion_rs_b200.attn as A  # noqa: E402
import nyion_rs_b200.splitkv as S  # noqa: E402
import oracle as O  # noqa: E402

N_KV, D, PT, H = 4, 64, 16, 32


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60))
    dev = torch.device("cuda")
    T = 20000
    rng = np.random.default_rng(99)
    src = rng.standard_normal((T, N_KV, 2, D), dtype=np.float32)
    q4 = O.q4_quantize_rows(src, D)
    q = rng.standard_normal((1, H, D), dtype=np.float32)
    decs = {m: S.SplitKVDecoder(rank, world, T, mode=m) for m in ("p2p", "collective")}
    dec = decs["p2p"]
    first, last = dec.lo // PT, (dec.hi + PT - 1) // PT
    local = np.zeros((last - first, N_KV, 2, PT, 40), np.uint8)
    for t in range(first * PT, min(last * PT, T)):
        local[t // PT - first, :, :, t % PT] = q4[t]
    table = np.zeros((1, (T + PT - 1) // PT), np.int32)
    table[0, first:last] = np.arange(last - first, dtype=np.int32)
    dq, dl, dt = torch.from_numpy(q).to(dev), torch.from_numpy(local).to(dev), torch.from_numpy(table).to(dev)
    outs = {}
    for m, d in decs.items():
        for _ in range(3):                       # consecutive steps alternate the mailbox halves
            outs[m] = d.step(dq, dl, dt).clone()
    # p2p steps replayed from a CUDA graph
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            gout = dec.step(dq, dl, dt, stream=s)
        for _ in range(4):
            g.replay()
    s.synchronize()
    outs["p2p-graph"] = gout.clone()
    del g
    out = outs["p2p"]
    torch.cuda.synchronize()
    # one-GPU reference on the full pool, and the oracle
    full = np.zeros(((T + PT - 1) // PT, N_KV, 2, PT, 40), np.uint8)
    for t in range(T):
        full[t // PT, :, :, t % PT] = q4[t]
    ftab = np.arange(full.shape[0], dtype=np.int32)[None]
    whole = A.lse_combine(A.decode_q4_partial(torch.from_numpy(q).to(dev), torch.from_numpy(full).to(dev),
                                              torch.from_numpy(ftab).to(dev), u_begin=0, u_end=T)[None])
    ref = O.lse_combine(O.decode_q4_partial(q, full, ftab, 0, T, N_KV, D, PT, threads=8)[None])
    for m, o in outs.items():
        err_gpu = (o - whole).abs().max().item()
        err_ref = np.abs(o.cpu().numpy() - ref).max()
        print(f"rank {rank}/{world} {m}: range [{dec.lo},{dec.hi}) vs one-GPU {err_gpu:.2e} vs oracle {err_ref:.2e}",
              flush=True)
        assert err_gpu < 1e-4 and err_ref < 1e-3
    assert A.device_error() == 0
    for d in decs.values():
        d.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
