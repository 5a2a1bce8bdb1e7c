"""GPU parity of the tensor-parallel gathered forward (obn_bitlinear_forward_tp).

One GPU: three "ranks" are three row-slice layers on the same device writing
into three output buffers through the per-rank (peer-store) form; every buffer
must equal the unsplit layer's forward bit for bit. Two or more GPUs: one
process per GPU over NCCL, outputs in symmetric memory, both the NVLS multicast
form (when the group has a multicast address) and the peer-store form, checked
on every rank against the unsplit forward computed locally.
"""
import datetime
import socket

import numpy as np
import pytest

from _util import need_cuda, obn, synth

pytestmark = pytest.mark.gpu


def tp():
    import importlib
    return importlib.import_module("0xbitnet_b200.tp")


@pytest.mark.parametrize("M,K,n", [(3000, 1024, 40), (3000, 1024, 300), (2560, 2560, 16),
                                   (9216, 3072, 129)])
def test_tp_peer_form_on_one_gpu_matches_unsplit(M, K, n):
    torch = need_cuda()
    world = 3
    L = synth().layer(31 + n, M, K)
    full = obn().BitLinear.from_i2s(L.blob(), K, M, norm_weight=L.gamma)
    x = torch.from_numpy(synth().activations(32 + n, n, K)).cuda()
    want = full.forward(x).cpu().numpy()
    parts = [tp().TPBitLinear(L.blob(), K, M, world, r, norm_weight=L.gamma) for r in range(world)]
    bufs = [torch.full((n, M), float("nan"), device="cuda") for _ in range(world)]
    ptrs = [b.data_ptr() for b in bufs]
    for p in parts:
        p.layer.forward_tp(x, M, p.row0, out_ranks=ptrs, n=n)
    torch.cuda.synchronize()
    for b in bufs:
        assert np.array_equal(b.cpu().numpy(), want)
    obn().check_device_errors()


def test_tp_argument_checks():
    torch = need_cuda()
    M, K = 512, 256
    L = synth().layer(3, M, K)
    part = tp().TPBitLinear(L.blob(), K, M, 2, 1)
    buf = torch.zeros((32, M), device="cuda")
    x = torch.zeros((32, K), device="cuda")
    E = obn()._lib
    with pytest.raises(E.ObnError) as ei:  # decode sizes are not served by the gathered form
        part.layer.forward_tp(x[:8], M, part.row0, out_ranks=[buf.data_ptr()], n=8)
    assert ei.value.code == E.OBN_ERR_UNSUPPORTED
    with pytest.raises(E.ObnError) as ei:  # columns past the output
        part.layer.forward_tp(x, M - 1, part.row0, out_ranks=[buf.data_ptr()], n=32)
    assert ei.value.code == E.OBN_ERR_INVALID_ARGUMENT


def _nccl_worker(rank, world, port, result_path):
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=120))
    results = []
    try:
        for (M, K, n) in [(9216, 3072, 256), (3000, 1024, 40)]:
            L = synth().layer(41 + n, M, K)
            full = obn().BitLinear.from_i2s(L.blob(), K, M, norm_weight=L.gamma, device=rank)
            x = torch.from_numpy(synth().activations(42 + n, n, K)).to(dev)
            want = full.forward(x)
            part = tp().TPBitLinear(L.blob(), K, M, world, rank, norm_weight=L.gamma,
                                    device=rank)
            out = tp().GatherOutput(n, M, device=dev)
            for mc in ([True, False] if out.mc_ptr else [False]):
                out.view(n).fill_(float("nan"))
                out.barrier()
                part.forward(x, out, multicast=mc)
                out.barrier()
                torch.cuda.synchronize()
                results.append(bool(torch.equal(out.view(n), want)))
            dist.barrier()
            part.close()
            full.close()
            del out
        obn().check_device_errors()
        ok = torch.tensor([1 if all(results) else 0], device=dev)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        if rank == 0:
            with open(result_path, "w") as f:
                f.write(f"{int(ok.item())} {len(results)}")
    finally:
        dist.destroy_process_group()


def test_tp_gather_across_gpus(tmp_path):
    torch = need_cuda()
    world = min(torch.cuda.device_count(), 8)
    if world < 2:
        pytest.skip("needs two or more GPUs")
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    path = str(tmp_path / "ok")
    mp.start_processes(_nccl_worker, args=(world, port, path), nprocs=world,
                       start_method="spawn", join=True)
    ok, count = open(path).read().split()
    assert ok == "1" and int(count) >= 2
