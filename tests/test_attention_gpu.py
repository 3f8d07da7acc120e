"""GPU parity of paged decode attention (tk_paged_attention; PagedAttention.forward,
src/kernels/attention.zig:51-100, shader src/kernels/shaders.zig:503-587).

Caches [block][heads][16][head_dim] with shuffled physical blocks per sequence, context lengths
that end inside a block, at a block boundary, and empty; head_dim 128, 64 and 80 (not a multiple
of 32).  Outputs against the f64 oracle, normwise 1e-5 (f32 accumulation, merged per warp).
"""
import numpy as np
import pytest

import oracle
from helpers import host
from tiny_kernel import _lib, ops

pytestmark = pytest.mark.gpu


def _case(seed, batch, heads, head_dim, ctxs, max_blocks):
    rng = np.random.default_rng(seed)
    nphys = batch * max_blocks + 3
    q = rng.standard_normal((batch, heads, head_dim)).astype(np.float32)
    kc = rng.standard_normal((nphys, heads, 16, head_dim)).astype(np.float32)
    vc = rng.standard_normal((nphys, heads, 16, head_dim)).astype(np.float32)
    bt = rng.permutation(nphys)[:batch * max_blocks].astype(np.int32).reshape(batch, max_blocks)
    cl = np.array(ctxs, dtype=np.int32)
    return q, kc, vc, bt, cl


@pytest.mark.parametrize("batch,heads,head_dim,ctxs,max_blocks", [
    (2, 8, 128, [37, 300], 20),
    (3, 4, 64, [16, 1, 0], 2),
    (1, 32, 128, [2048], 128),
    (2, 6, 80, [95, 160], 10),
])
def test_paged_attention_vs_oracle(torch_cuda, tkdev, batch, heads, head_dim, ctxs, max_blocks):
    torch = torch_cuda
    q, kc, vc, bt, cl = _case(batch * 100 + head_dim, batch, heads, head_dim, ctxs, max_blocks)
    d = [torch.from_numpy(a).cuda() for a in (q, kc, vc, bt, cl)]
    o = torch.empty((batch, heads, head_dim), dtype=torch.float32, device="cuda")
    ops.paged_attention(tkdev, *d, o, batch, heads, head_dim, max_blocks)
    ref = oracle.paged_attention_f64(q, kc, vc, bt, cl, batch, heads, head_dim, max_blocks)
    y = host(o)
    assert np.all(y[np.array(ctxs) == 0] == 0)
    assert oracle.normwise_err(y, ref) <= 1e-5


def test_paged_attention_rejects_bad_shapes(torch_cuda, tkdev):
    L = _lib.lib()
    t = torch_cuda.zeros(16, device="cuda")
    p = t.data_ptr()
    assert L.tk_paged_attention(tkdev.handle, p, p, p, p, p, p, 1, 1, 129, 1) == _lib.TK_ERR_ARG
    assert L.tk_paged_attention(tkdev.handle, p, p, p, p, p, p, 0, 1, 64, 1) == _lib.TK_ERR_ARG
    assert L.tk_paged_attention(tkdev.handle, None, p, p, p, p, p, 1, 1, 64, 1) == _lib.TK_ERR_ARG
