"""Regenerates the golden fixtures in this directory from the CPU oracle.

    python tests/golden/make_golden.py

Each fixture stores seeded inputs (or a sha256 of inputs regenerated from the
seed by 0xbitnet_b200.synthetic) together with the oracle's outputs: q (int8),
scales, qsum, int32 accumulators and float32 y. The oracle (oracle/) restates
the reference's WGSL kernels and is itself pinned by tests/test_oracle_kat.py.
"""
import importlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import oracle as orc  # noqa: E402

synth = importlib.import_module("0xbitnet_b200.synthetic")
i2s = importlib.import_module("0xbitnet_b200.i2s")


def sha(*arrays):
    import hashlib
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def seeded_case(name, seed, n, M, K, norm):
    L = synth.layer(seed, M, K)
    x = synth.activations(seed + 1, n, K)
    gamma = L.gamma if norm else None
    y, q, s = orc.bitlinear(x, L.packed, L.row_scales(), M, K, norm_w=gamma)
    acc = orc.ternary_acc(L.packed, q, M, K)
    np.savez_compressed(
        os.path.join(HERE, f"{name}.npz"), seed=seed, n=n, M=M, K=K, norm=norm,
        inputs_sha=sha(L.packed, np.float32(L.scale), L.gamma, x),
        q=q, scales=s, qsum=q.astype(np.int64).sum(1).astype(np.int32), acc=acc, y=y)


def kat_gemv():
    # ternary-gemv.test.ts:13-26 setup(seed=42): M=8, K=256.
    M, K = 8, 256
    rows = np.stack([orc.rand_ternary(K, 42 + m) for m in range(M)])
    packed = orc.i2s_pack_matrix(rows)
    q = orc.rand_int8(K, 142).astype(np.int8)
    s_w = np.array([0.01 + 0.001 * m for m in range(M)], np.float32)
    y = orc.ternary_gemv(packed, q, s_w, np.float32(0.05), M, K)
    np.savez_compressed(os.path.join(HERE, "kat_gemv_seed42.npz"), packed=packed, q=q, s_w=s_w,
                        s_x=np.float32(0.05), y=y, acc=orc.ternary_acc(packed, q, M, K))


def kat_gemm():
    # ternary-gemm.test.ts:37-72 (output layout): M=4, K=128, N=3.
    M, K, N = 4, 128, 3
    packed = orc.i2s_pack_matrix(np.stack([orc.rand_ternary(K, 20 + m) for m in range(M)]))
    q = orc.rand_int8(N * K, 200).astype(np.int8).reshape(N, K)
    s_w = np.full(M, 0.01, np.float32)
    s_x = np.array([0.01 + 0.005 * n for n in range(N)], np.float32)
    y = orc.ternary_gemm(packed, q, s_w, s_x, M, K)
    np.savez_compressed(os.path.join(HERE, "kat_gemm_layout.npz"), packed=packed, q=q, s_w=s_w,
                        s_x=s_x, y=y, acc=orc.ternary_acc(packed, q, M, K))


def kat_e2e():
    # bitlinear-e2e.test.ts:111-139 (GEMV matches GEMM, N=1): K=256, M=128, randf32(256, 10).
    K, M = 256, 128
    x = orc.randf32(K, 10)[None]
    packed = orc.i2s_pack_matrix(np.stack([orc.rand_ternary(K, 100 + i) for i in range(M)]))
    y, q, s = orc.bitlinear(x, packed, np.ones(M, np.float32), M, K)
    np.savez_compressed(os.path.join(HERE, "kat_e2e_n1.npz"), x=x, packed=packed, y=y, q=q,
                        scales=s)


if __name__ == "__main__":
    seeded_case("cfg0_fused_gemv", 1234, 1, 2560, 2560, True)
    seeded_case("cfg1_o_b8", 2025, 8, 2560, 2560, True)
    seeded_case("cfg1_down_b3_nonorm", 77, 3, 2560, 6912, False)
    kat_gemv()
    kat_gemm()
    kat_e2e()
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)))
