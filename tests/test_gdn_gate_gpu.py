"""Parity of q35_gdn_gate (beta / g) against the oracle: mode 0 follows
kernels.rs:174-247 (decode; the cluster kernel and the one-CTA kernel for
splits too large to stage), mode 1 text_modules.rs:578-595 (prefill)."""
import numpy as np
import pytest
import torch

import oracle
import q35attn
from conftest import max_rel_err

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("mode,N,H,ind", [
    (0, 1, 16, 2048), (0, 5, 16, 2048), (1, 300, 16, 2048), (1, 7, 32, 2048), (1, 9, 2, 2048), (0, 3, 2, 2048),
    (0, 1, 64, 2048),   # 128 KB of staged weights per split
    (0, 2, 48, 4096),   # 196 KB: the largest split that is staged
    (0, 1, 64, 4096),   # too large to stage: the one-CTA kernel
    (0, 2, 16, 1000),   # chunk 125: the reference walks 120 rows per split; unaligned rows
    (0, 1, 16, 40),     # fewer than 8 rows per split
])
def test_gate(mode, N, H, ind):
    rng = np.random.RandomState(mode * 100 + N + H + ind)
    x = rng.randn(N, ind).astype(np.float32)
    wb = (0.02 * rng.randn(ind, H)).astype(np.float32)
    wa = (0.02 * rng.randn(ind, H)).astype(np.float32)
    a_log = np.log(rng.uniform(0.01, 16.0, H)).astype(np.float32)
    dt = np.ones(H, np.float32)
    T = lambda a: torch.from_numpy(a).cuda()
    beta, g = q35attn.gdn_gate(T(x), T(wb), T(wa), T(a_log), T(dt), mode=mode)
    rb, rg = oracle.gate_proj(x, wb, wa, a_log, dt, mode=mode)
    assert max_rel_err(beta.cpu().numpy(), rb) <= 1e-5
    assert max_rel_err(g.cpu().numpy(), rg) <= 1e-5
