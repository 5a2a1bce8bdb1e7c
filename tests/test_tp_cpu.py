"""Tensor-parallel (output-feature split) host logic, on CPU.

The gathered forward splits an out_total-row BitLinear into contiguous row
blocks, one per rank; every rank computes its block and the blocks land side by
side in each rank's [n, out_total] output. These tests check, with the oracle
standing in for the GPU, that the row split covers every row once, that a row
slice of an I2_S tensor is an I2_S tensor of its own, and — over a world_size-2
gloo group — that gathering the ranks' slices rebuilds the unsplit layer's
output exactly. The C-ABI entry point's argument checks run without a GPU.
"""
import ctypes
import os
import socket

import numpy as np
import pytest

import oracle as orc
from _util import obn, synth


def tp():
    import importlib
    return importlib.import_module("0xbitnet_b200.tp")


@pytest.mark.parametrize("out_dim", [1, 7, 128, 2560, 3000, 9216])
@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_row_ranges_partition_rows(out_dim, world):
    if world > out_dim:
        pytest.skip("more ranks than rows")
    ranges = [tp().row_range(out_dim, world, r) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == out_dim
    for (a0, a1), (b0, b1) in zip(ranges, ranges[1:]):
        assert a1 == b0 and a0 < a1
    sizes = [b - a for a, b in ranges]
    assert max(sizes) - min(sizes) <= 1


def test_row_slice_is_an_i2s_tensor():
    M, K = 300, 256
    L = synth().layer(5, M, K)
    blob = L.blob()
    part = tp().slice_i2s_rows(blob, K, M, 100, 220)
    rows, scale = obn().i2s.split_tensor(part, K, 120)
    full_rows, full_scale = obn().i2s.split_tensor(blob, K, M)
    assert scale == full_scale
    assert np.array_equal(rows, full_rows[100:220])
    with pytest.raises(ValueError):
        tp().slice_i2s_rows(blob, K, M, 200, 301)


def _slice_forward(L, x, M, K, world, rank):
    r0, r1 = tp().row_range(M, world, rank)
    part = tp().slice_i2s_rows(L.blob(), K, M, r0, r1)
    rows, scale = obn().i2s.split_tensor(part, K, r1 - r0)
    y, _, _ = orc.bitlinear(x, rows, np.full(r1 - r0, scale, np.float32), r1 - r0, K,
                            norm_w=L.gamma)
    return r0, y


def test_slices_concatenate_to_the_full_layer():
    M, K, n = 1000, 384, 5
    L = synth().layer(11, M, K)
    x = synth().activations(12, n, K)
    full, _, _ = orc.bitlinear(x, L.packed, L.row_scales(), M, K, norm_w=L.gamma)
    for world in (2, 3, 7):
        out = np.zeros_like(full)
        for r in range(world):
            r0, y = _slice_forward(L, x, M, K, world, r)
            out[:, r0:r0 + y.shape[1]] = y
        assert np.array_equal(out, full)


def _gloo_worker(rank, world, port, result_path):
    import torch
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    try:
        M, K, n = 515, 256, 3
        L = synth().layer(21, M, K)
        x = synth().activations(22, n, K)
        r0, y = _slice_forward(L, x, M, K, world, rank)
        # all ranks exchange (col0, slice) and assemble the gathered output
        parts = [None] * world
        dist.all_gather_object(parts, (r0, y))
        out = np.zeros((n, M), np.float32)
        for c0, ys in parts:
            out[:, c0:c0 + ys.shape[1]] = ys
        full, _, _ = orc.bitlinear(x, L.packed, L.row_scales(), M, K, norm_w=L.gamma)
        ok = torch.tensor([1 if np.array_equal(out, full) else 0])
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        if rank == 0:
            with open(result_path, "w") as f:
                f.write(str(int(ok.item())))
    finally:
        dist.destroy_process_group()


def test_gather_over_gloo_world2(tmp_path):
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    path = str(tmp_path / "ok")
    mp.start_processes(_gloo_worker, args=(2, port, path), nprocs=2, start_method="spawn",
                       join=True)
    assert open(path).read() == "1"


def test_forward_tp_rejects_bad_arguments_without_a_device():
    lib = obn().lib()
    E = obn()._lib
    buf = ctypes.c_void_p(16)
    # null layer
    assert lib.obn_bitlinear_forward_tp(None, buf, 16, buf, None, 1, 16, 0, buf, 1 << 20,
                                        None) == E.OBN_ERR_INVALID_ARGUMENT
    assert b"NULL" in lib.obn_error_message()
