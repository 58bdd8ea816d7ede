"""Vocab-parallel CE as two real ranks: separate processes, a gloo process group.

Both ranks run their kernels on cuda:0 (each process has its own context; no
kernel waits on another rank's kernel) and the collectives of
vocab_parallel_cross_entropy go through gloo on host copies of the device
buffers: the all-gather of the per-token records and the reduce-scatter of the
bf16 partial dhidden over token blocks (or the fp32 all-reduce). Each rank
checks its results against the CPU oracle on the full vocabulary.
"""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

N, V, D = 300, 20011, 256  # rows not a multiple of the rank count, ragged vocab


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    g = torch.Generator().manual_seed(31)
    hidden = torch.randn(N, D, generator=g).to(torch.bfloat16)
    weight = (0.02 * torch.randn(V, D, generator=g)).to(torch.bfloat16)
    targets = torch.randint(0, V, (N,), generator=g)
    logits = hidden.float() @ weight.float().t()
    plant = torch.rand(N, generator=g) < 0.3
    targets[plant] = logits.argmax(-1)[plant]  # hits far from zero
    targets[torch.rand(N, generator=g) < 0.1] = -100
    targets[7] = V - 1
    targets[8] = 0
    return hidden, weight, targets, logits


def _rank_main(rank, world, port, mode, out_dir):
    import torch.distributed as dist

    import oracle
    from auspex_soup_demo_b200 import _lib
    from auspex_soup_demo_b200.kernels.vocab_parallel import (shard_range, token_block,
                                                              vocab_parallel_cross_entropy)
    from helpers import cosine

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    ok = False
    try:
        torch.cuda.set_device(0)
        hidden, weight, targets, logits = _inputs()
        den = float((targets != -100).sum())
        loss, ent, corr, grad, _ = oracle.ce_rows(logits, targets, den)
        dh_ref = grad @ weight.float()
        off, size = shard_range(V, rank, world)
        dw_ref = grad[:, off:off + size].t() @ hidden.float()
        losses, ents, hits, sums, dh, dw = vocab_parallel_cross_entropy(
            hidden.cuda(), weight[off:off + size].cuda(), off, V, targets.cuda(), den,
            dh_reduce=mode)
        torch.cuda.synchronize()
        assert _lib.device_error(torch.device("cuda", 0)) == 0
        torch.testing.assert_close(losses.cpu(), loss, rtol=1e-4, atol=1e-4)
        torch.testing.assert_close(ents.cpu(), ent, rtol=2e-3, atol=2e-3)
        assert torch.equal(hits.cpu(), corr)
        assert int(corr.sum()) > 50
        assert abs(float(sums[0]) - float(loss.sum())) <= 1e-4 * float(loss.sum())
        if mode == "scatter":
            start, count = token_block(N, rank, world)
            assert dh.shape == (count, D) and dh.dtype == torch.bfloat16
            assert cosine(dh, dh_ref[start:start + count]) >= 0.9999
        else:
            assert dh.shape == (N, D) and dh.dtype == torch.float32
            assert cosine(dh, dh_ref) >= 0.9999
        assert cosine(dw, dw_ref) >= 0.9999
        ok = True
    finally:
        with open(os.path.join(out_dir, f"rank{rank}.{'ok' if ok else 'fail'}"), "w"):
            pass
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["scatter", "all"])
def test_vocab_parallel_two_gloo_ranks(mode, tmp_path):
    world = 2
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, mode, str(tmp_path)))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
    codes = [p.exitcode for p in procs]
    assert codes == [0, 0], codes
    for r in range(world):
        assert (tmp_path / f"rank{r}.ok").exists(), f"rank {r} failed"
