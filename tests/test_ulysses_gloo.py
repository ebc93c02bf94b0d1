"""The sequence-parallel (Ulysses) data movement of the step, on 2 gloo ranks on the CPU: each rank packs its rows'
q/k/v into the send layout the q/k/v epilogue writes ([P][S_l][3][H/P][128]), exchanges with every peer, runs
attention for its heads over the whole sequence, sends the output back and applies the out projection to the
received chunks read as a column-chunked A ([P][S_l][H/P x 128]), exactly as the library lays them out. The result
must equal the single-process computation (and padding rows at the end of the last rank must not change it)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import h3_oracle as O


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def exchange(send, P):
    """send [P][chunk...] -> recv [P][chunk...]: block r goes to rank r (grouped point-to-point, like the NCCL calls)."""
    recv = torch.empty_like(send)
    reqs = []
    me = dist.get_rank()
    for r in range(P):
        if r == me:
            recv[r] = send[r]
            continue
        reqs.append(dist.isend(send[r].contiguous(), r))
        reqs.append(dist.irecv(recv[r], r))
    for q in reqs:
        q.wait()
    return recv


def worker(rank, P, port, S, H, d, out_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=P)
    g = torch.Generator().manual_seed(0)
    qkv_full = torch.randn(S, 3, H, 128, generator=g)
    Wout = torch.randn(d, H * 128, generator=g) * 0.05
    Sl = (S + P - 1) // P
    Hp = H // P
    rows = torch.zeros(Sl, 3, H, 128)
    lo, hi = rank * Sl, min(S, rank * Sl + Sl)
    rows[:hi - lo] = qkv_full[lo:hi]
    # the q/k/v epilogue's send layout: [P][S_l][3][H/P][128], block r holding heads r*Hp .. r*Hp+Hp-1
    send = rows.reshape(Sl, 3, P, Hp, 128).permute(2, 0, 1, 3, 4).contiguous()
    recv = exchange(send, P).reshape(P * Sl, 3, Hp, 128)  # [S_pad][3][H/P][128]: the whole sequence, my heads
    # attention over the valid rows only (keys past S are masked by the kernel's row bound)
    o = torch.zeros(P * Sl, Hp, 128)
    o[:S] = O.attention(recv[:S, 0], recv[:S, 1], recv[:S, 2])
    back = exchange(o.reshape(P, Sl, Hp * 128).contiguous(), P)  # [P][S_l][Hp*128]: my rows, every rank's heads
    A = back.permute(1, 0, 2).reshape(Sl, H * 128)  # the chunked A read as one [S_l][inner] matrix
    y = A @ Wout.T
    out_q.put((rank, y[:hi - lo].numpy()))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("S", [96, 101])
def test_ulysses_two_gloo_ranks_match_single_process(S):
    P, H, d = 2, 4, 64
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=worker, args=(r, P, port, S, H, d, q)) for r in range(P)]
    for p in procs:
        p.start()
    parts = dict(q.get(timeout=120) for _ in range(P))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    got = np.concatenate([parts[r] for r in range(P)])
    g = torch.Generator().manual_seed(0)
    qkv_full = torch.randn(S, 3, H, 128, generator=g)
    Wout = torch.randn(d, H * 128, generator=g) * 0.05
    want = (O.attention(qkv_full[:, 0], qkv_full[:, 1], qkv_full[:, 2]).reshape(S, H * 128) @ Wout.T).numpy()
    np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-4)
