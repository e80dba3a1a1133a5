"""KV-head sharding (``autoindexer_b200.sharding``): each rank computes the
query heads of its KV heads and the results are all-gathered by head.

CPU, gloo, world size 2: the oracle stands in for the local attention, and
the gathered forward output and gradients must equal the unsharded oracle's
exactly (a GQA group's heads depend on nothing outside the group).  GPU: the
kernel path with one rank equals ``AttentionFn`` bit for bit, and with two
GPUs (NCCL; skipped when fewer are visible) the gathered results equal each
rank's unsharded run bit for bit.
"""

import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from conftest import ROOT


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _case(T=96, Hq=8, Hkv=2, D=32, seed=7):
    """Two documents per row, two RoPE sections; float64 inputs."""
    sys.path.insert(0, ROOT)
    from autoindexer_b200 import RowLayouts, SectionedRope, cursor_stream, document_blocks
    from oracle import attn_oracle as O

    rng = np.random.default_rng(seed)
    streams = [np.arange(T), cursor_stream(T, rng)]
    sections = [(0, D // 4), (D // 4, D // 2)]
    mod = SectionedRope(D, 1e6, [torch.as_tensor(s) for s in streams], sections)
    rope = O.make_sectioned_rope(mod.inv_freq.numpy(), streams, sections)
    rows = RowLayouts()
    rows.append(document_blocks([T // 3, T - T // 3], position_ids=np.arange(T)))
    q, k, v = (rng.standard_normal(s) for s in ((1, Hq, T, D), (1, Hkv, T, D), (1, Hkv, T, D)))
    dout = rng.standard_normal((1, T, Hq, D))
    return rows, mod, rope, q, k, v, dout


def _oracle_local(rope):
    """Local forward / backward of one rank's heads by the oracle, writing
    into the buffer views the sharded path hands over."""
    from oracle import attn_oracle as O

    def fwd(q, k, v, rows, scale, out_bhtd=None):
        out, _ = O.attn_forward(q.detach().numpy(), k.detach().numpy(), v.detach().numpy(), rows, rope, scale)
        out = torch.from_numpy(out)
        if out_bhtd is not None:
            out_bhtd.copy_(out.permute(0, 2, 1, 3))
        return out, (q, k, v, rows, scale)

    def bwd(state, dout, grads=None, after_dq=None):
        # dQ is written first and handed over (its gather starts) before dK and dV
        q, k, v, rows, scale = state
        res = O.attn_backward(q.detach().numpy(), k.detach().numpy(), v.detach().numpy(), dout.numpy(), rows,
                              rope, scale)
        res = tuple(torch.from_numpy(x) for x in res)
        if grads is not None:
            grads[0].copy_(res[0])
            if after_dq is not None:
                after_dq()
            for g, x in zip(grads[1:], res[1:]):
                g.copy_(x)
        elif after_dq is not None:
            after_dq()
        return res

    return fwd, bwd


def _gloo_rank(rank: int, world: int, port: int, out):
    sys.path.insert(0, ROOT)
    import torch.distributed as dist

    from autoindexer_b200.sharding import kv_sharded_attention

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rows, _, rope, q, k, v, dout = _case()
        fwd, bwd = _oracle_local(rope)
        tq, tk, tv = (torch.from_numpy(x).requires_grad_(True) for x in (q, k, v))
        scale = q.shape[-1] ** -0.5
        o = kv_sharded_attention(tq, tk, tv, list(rows), scale, None, fwd, bwd, overlap=True)
        o.backward(torch.from_numpy(dout))
        out.put((rank, o.detach().numpy(), tq.grad.numpy(), tk.grad.numpy(), tv.grad.numpy()))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_ranks_gather_equals_unsharded_oracle():
    from oracle import attn_oracle as O

    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q_ = ctx.Queue()
    procs = [ctx.Process(target=_gloo_rank, args=(r, world, port, q_)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, *vals = q_.get(timeout=180)
        res[r] = vals
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    rows, _, rope, q, k, v, dout = _case()
    out, _ = O.attn_forward(q, k, v, list(rows), rope)
    dq, dk, dv = O.attn_backward(q, k, v, dout, list(rows), rope)
    for r in range(world):
        for got, want in zip(res[r], (out, dq, dk, dv)):
            np.testing.assert_array_equal(got, want)


def test_head_range_rejects_uneven_split():
    sys.path.insert(0, ROOT)
    from autoindexer_b200.sharding import head_range

    assert head_range(8, 1, 4) == (2, 4)
    with pytest.raises(ValueError):
        head_range(8, 0, 3)


def _bf16_inputs(device, B=1, T=640, Hq=8, Hkv=4, D=128, seed=11):
    rows, mod, _, *_ = _case(T=T, Hq=Hq, Hkv=Hkv, D=D, seed=seed)
    g = torch.Generator().manual_seed(seed)
    q, k, v = (torch.randn(B, h, T, D, generator=g).to(torch.bfloat16).to(device) for h in (Hq, Hkv, Hkv))
    dout = torch.randn(B, T, Hq, D, generator=g).to(torch.bfloat16).to(device)
    return rows, mod, q, k, v, dout


def _run(fn, q, k, v, dout):
    xs = [x.detach().clone().requires_grad_(True) for x in (q, k, v)]
    o = fn(*xs)
    o.backward(dout)
    return [o.detach()] + [x.grad for x in xs]


@pytest.mark.gpu
def test_one_rank_kernel_path_equals_attention_fn(cuda_device):
    from autoindexer_b200 import AttentionFn, compile_layout
    from autoindexer_b200.sharding import kv_sharded_attention

    rows, mod, q, k, v, dout = _bf16_inputs(cuda_device)
    lay = compile_layout(rows, 1, q.shape[2], 128, torch.bfloat16, mod.to(cuda_device), cuda_device)
    sc = 128 ** -0.5
    a = _run(lambda x, y, z: kv_sharded_attention(x, y, z, lay, sc), q, k, v, dout)
    b = _run(lambda x, y, z: AttentionFn.apply(x, y, z, lay, sc), q, k, v, dout)
    for x, y in zip(a, b):
        assert torch.equal(x, y)


def _nccl_rank(rank: int, world: int, port: int, out):
    sys.path.insert(0, ROOT)
    import torch.distributed as dist

    from autoindexer_b200 import AttentionFn, compile_layout
    from autoindexer_b200.sharding import kv_sharded_attention

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      NCCL_NVLS_ENABLE="0")
    from datetime import timedelta

    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        rows, mod, q, k, v, dout = _bf16_inputs(dev)
        lay = compile_layout(rows, 1, q.shape[2], 128, torch.bfloat16, mod.to(dev), dev)
        sc = 128 ** -0.5
        a = _run(lambda x, y, z: kv_sharded_attention(x, y, z, lay, sc), q, k, v, dout)
        b = _run(lambda x, y, z: AttentionFn.apply(x, y, z, lay, sc), q, k, v, dout)
        c = _run(lambda x, y, z: kv_sharded_attention(x, y, z, lay, sc, overlap=True), q, k, v, dout)
        torch.cuda.synchronize(dev)
        out.put((rank, all(torch.equal(x, y) and torch.equal(x, w) for x, y, w in zip(a, b, c))))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_two_gpus_nccl_gather_equals_unsharded(cuda_device):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q_ = ctx.Queue()
    procs = [ctx.Process(target=_nccl_rank, args=(r, world, port, q_)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q_.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert got == {0: True, 1: True}
