"""The peer-memory exchange of the tensor-parallel decoder (``iron_peer_exchange``,
``iron_b200.tp.PeerCollective``) on two GPUs, one process per GPU (spawned here; the
test is skipped with fewer than two GPUs, since the kernel of one rank waits for the
other's and two ranks must never share a GPU).  Checked: the float32 sum in rank order
and the gather, against the inputs; many calls in a row and replays of a captured CUDA
graph (the slots alternate by the device-side epoch); a 2-layer Qwen3 tensor-parallel
step with the peer exchange gives the tokens and logits of the same step over NCCL."""

import datetime
import os
import socket
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, outdir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    res = {}
    try:
        from iron_b200.qwen3 import Qwen3Config, Qwen3Weights
        from iron_b200.tp import PeerCollective, Qwen3TP
        n = 4096
        pc = PeerCollective(world, rank, n, dev)
        g = torch.Generator(device=dev).manual_seed(100 + rank)
        # sums and gathers, alternating, 50 calls
        ok_sum = ok_gather = True
        for it in range(25):
            x = torch.randn(n, generator=g, device=dev)
            allx = [torch.empty_like(x) for _ in range(world)]
            dist.all_gather(allx, x)
            want = torch.zeros_like(x)
            for r in range(world):
                want += allx[r]
            y = x.clone()
            pc(("sum", y))
            ok_sum &= torch.equal(y, want)
            pairs = torch.tensor([[rank * 10 + it, it]], dtype=torch.int32, device=dev)
            got = torch.empty(world, 1, 2, dtype=torch.int32, device=dev)
            pc(("gather", got, pairs))
            ok_gather &= all(int(got[r, 0, 0]) == r * 10 + it and int(got[r, 0, 1]) == it for r in range(world))
        res["sum"], res["gather"] = ok_sum, ok_gather
        # a captured graph of 3 sums, replayed 10 times
        xs = torch.randn(n, generator=g, device=dev)
        buf = xs.clone()
        st = torch.cuda.Stream(device=dev)
        st.wait_stream(torch.cuda.current_stream())
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=st):
            for _ in range(3):
                pc(("sum", buf))
        allx = [torch.empty_like(xs) for _ in range(world)]
        dist.all_gather(allx, xs)
        ok_graph = True
        for _ in range(10):
            buf.copy_(xs)
            torch.cuda.synchronize()
            gr.replay()
            torch.cuda.synchronize()
            # the first sum gives S on every rank, the next two world * S and world^2 * S
            ok_graph &= torch.allclose(buf, sum(allx) * world ** 2, rtol=1e-6, atol=1e-5)
        res["graph"] = ok_graph
        res["err"] = int(pc.err.item())
        del gr
        # a 2-layer Qwen3 step: peer exchange vs NCCL
        cfg = Qwen3Config.qwen3_0_6b()
        w = Qwen3Weights.synthetic(cfg, seed=4, group=32, n_layers=2, device=dev)
        toks = {}
        for coll in ("nccl", "peer"):
            dec = Qwen3TP(w, rank, world, max_seq=64, batch=1, device=dev, collective=coll)
            out = []
            t = [17]
            for pos in range(6):
                t = [int(v) for v in dec.step_tokens(t, pos)]
                out.append((t[0], dec.logits[0].float().cpu()))
            dec.close()
            toks[coll] = out
        res["tp_tokens"] = [a[0] for a in toks["peer"]] == [a[0] for a in toks["nccl"]]
        res["tp_logits"] = all(torch.equal(a[1], b[1]) for a, b in zip(toks["peer"], toks["nccl"]))
    finally:
        torch.save(res, os.path.join(outdir, f"rank{rank}.pt"))
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="the peer exchange needs two GPUs (one per rank)")
def test_peer_exchange_two_gpus():
    world = 2
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_rank, args=(world, _free_port(), d), nprocs=world, join=True)
        for r in range(world):
            res = torch.load(os.path.join(d, f"rank{r}.pt"))
            assert res.get("sum") and res.get("gather"), res
            assert res.get("graph"), res
            assert res.get("err") == 0, res
            assert res.get("tp_tokens") and res.get("tp_logits"), res
