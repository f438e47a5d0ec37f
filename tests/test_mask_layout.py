"""CPU: the valid-first row layout a padding mask selects (host-side tables of the DiT workspace).

Rows [0, V) must hold, per sequence and in order, its memory tokens then its valid latents (the packed token
order of the reference's flash-varlen path, transformer.py:620-651); rows [V, M) the padded latents. RoPE
positions stay the original ones, and every latent maps to exactly one stream row.
"""
import numpy as np
import pytest
import torch

from sa3_b200.engine import _Workspace
from sa3_b200.modules import DiTConfig


@pytest.mark.parametrize("valid", [
    [np.arange(137), np.arange(200)],                  # a valid prefix and a full prompt
    [np.array([0, 3, 4, 9, 150]), np.arange(0, 200, 7)],  # arbitrary (non-prefix) masks
    [np.arange(0), np.arange(5)],                      # a prompt with no valid latent
])
def test_valid_first_tables(valid):
    cfg = DiTConfig(embed_dim=128, depth=1, num_heads=2, sliding_window=(8, 8), differential=False)
    L, nm = 200, cfg.num_memory_tokens
    ws = _Workspace(cfg, [L, L], 4, "cpu", fp8=False, valid=valid)
    B, M = 2, 2 * (L + nm)
    cu = ws.cu.numpy()
    assert ws.masked and ws.uniform_n == 0
    assert list(cu) == [0, nm + len(valid[0]), 2 * nm + len(valid[0]) + len(valid[1])]
    assert ws.V == cu[-1]
    rb, pos, lat = ws.row_batch.numpy(), ws.row_pos.numpy(), ws.lat_rows.numpy()
    # every stream row is a memory token or exactly one latent
    mem = ws.mem_rows.numpy()
    assert sorted(np.concatenate([mem, lat]).tolist()) == list(range(M))
    for b in range(B):
        r0 = cu[b]
        assert list(mem[b * nm:(b + 1) * nm]) == list(range(r0, r0 + nm))
        assert (pos[r0:r0 + nm] == np.arange(nm)).all()
        vi = valid[b]
        rows_v = lat[b * L + vi]
        assert list(rows_v) == list(range(r0 + nm, cu[b + 1]))          # packed, in order
        pi = np.setdiff1d(np.arange(L), vi)
        rows_p = lat[b * L + pi]
        assert (rows_p >= ws.V).all()
        assert (pos[lat[b * L:(b + 1) * L]] == nm + np.arange(L)).all()  # original positions
        assert (rb[lat[b * L:(b + 1) * L]] == b).all() and (rb[mem[b * nm:(b + 1) * nm]] == b).all()
    # padded segments for the cross-attention's second launch
    cp = ws.cu_pad.numpy()
    assert list(np.diff(cp)) == [L - len(v) for v in valid]
    for b in range(B):
        assert (rb[ws.V + cp[b]:ws.V + cp[b + 1]] == b).all()
    assert ws.max_n == nm + max(len(v) for v in valid)
    # self-attention output rows of padded tokens start (and stay) zero
    assert torch.count_nonzero(ws.o[ws.V:]) == 0 and ws.ox is not ws.o


def test_unmasked_layout_unchanged():
    cfg = DiTConfig(embed_dim=128, depth=1, num_heads=2, differential=False)
    ws = _Workspace(cfg, [50, 50], 4, "cpu", fp8=False)
    assert not ws.masked and ws.V == ws.M and ws.ox is ws.o and ws.uniform_n == 50 + cfg.num_memory_tokens
