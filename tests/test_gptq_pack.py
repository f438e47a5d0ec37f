"""CPU: GPTQ int4 packing — the oracle's pack/unpack round-trips, the product's unpack and repack agree
with it bit for bit (int4 index math must be bit-exact)."""
import numpy as np
import torch

from oracle import quant as oq
from sa3_b200 import gptq


def test_oracle_pack_unpack_roundtrip():
    rng = np.random.default_rng(0)
    K, N, G = 256, 64, 2
    q = rng.integers(0, 16, size=(K, N))
    z = rng.integers(0, 16, size=(G, N))
    s = rng.uniform(0.001, 0.02, size=(G, N))
    g_idx = rng.permutation(K) // 128
    qw, qz, sc, gi = oq.gptq_pack(q, z, s, g_idx)
    q2, z2 = oq.gptq_unpack(qw, qz)
    assert np.array_equal(q2, q) and np.array_equal(z2, z)


def test_product_unpack_matches_oracle():
    qw, qz, sc, gi = oq.random_gptq_layer(256, 512, seed=3)
    q1, z1 = oq.gptq_unpack(qw, qz)
    q2, z2 = gptq.unpack(qw, qz)
    assert np.array_equal(q1, q2) and np.array_equal(z1, z2)


def test_repack_layout_is_the_sorted_dequantised_weight():
    """Decode the kernel layout on the CPU and compare with the oracle's dequantised W[:, perm]."""
    qw, qz, sc, gi = oq.random_gptq_layer(128, 384, seed=5)
    p = gptq.repack(qw, qz, sc, gi)
    perm = p["perm"].numpy()
    words = p["qw"].numpy().view(np.uint32)  # [N, K/8]
    N, K8 = words.shape
    q = np.zeros((N, K8 * 8), dtype=np.int64)
    for j in range(8):
        q[:, j::8] = (words >> np.uint32(4 * j)) & 0xF
    sz = p["sz"].numpy()
    grp = np.arange(K8 * 8) // 128
    w_kernel = q * sz[grp, :N].T - sz[grp, N:].T  # q*s - z*s per (n, k')
    w_ref = oq.gptq_dequant(qw, qz, sc, gi)[:, perm]
    assert np.array_equal(w_kernel.astype(np.float32), w_ref.astype(np.float32))
