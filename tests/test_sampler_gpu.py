"""GPU parity of the sampler kernels: argmax and softmax_sample (src/kernels/shaders.zig:826-943;
the host sampler of src/model/llama.zig:290-323).

argmax: the index of the largest value, ties to the smallest index (the shader's tie rule
follows its thread layout and is not kept).  softmax_sample: probabilities within 1e-6 of the
f64 softmax (normwise, against the largest probability); the sampled index equal to the f64
search for random values placed midway between cumulative boundaries (the kernel's f32 sums run
in a different order than the shader's, which matters only within rounding of a boundary).
"""
import numpy as np
import pytest

import oracle
from helpers import host
from tiny_kernel import _lib, ops

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n", [1, 2, 1000, 32000, 128256])
def test_argmax(torch_cuda, tkdev, n):
    torch = torch_cuda
    x = np.random.default_rng(n).standard_normal(n).astype(np.float32) * 4
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops.argmax(tkdev, torch.from_numpy(x).cuda(), n, out)
    assert int(host(out)[0]) == oracle.argmax_ref(x)


def test_argmax_ties_and_infinities(torch_cuda, tkdev):
    torch = torch_cuda
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    x = np.zeros(5000, dtype=np.float32)
    x[[777, 3000, 4999]] = 2.5
    ops.argmax(tkdev, torch.from_numpy(x).cuda(), len(x), out)
    assert int(host(out)[0]) == 777
    x = np.full(300, -np.inf, dtype=np.float32)
    ops.argmax(tkdev, torch.from_numpy(x).cuda(), len(x), out)
    assert int(host(out)[0]) == 0


@pytest.mark.parametrize("n,temperature", [(32000, 1.0), (128256, 0.7), (7, 2.0), (1, 1.0)])
def test_softmax_sample(torch_cuda, tkdev, n, temperature):
    torch = torch_cuda
    logits = np.random.default_rng(n + 1).standard_normal(n).astype(np.float32) * 3
    ld = torch.from_numpy(logits).cuda()
    probs = torch.empty(n, dtype=torch.float32, device="cuda")
    sampled = torch.zeros(1, dtype=torch.int32, device="cuda")
    ref = oracle.softmax_f64(logits, temperature)
    c = np.cumsum(ref)
    rng = np.random.default_rng(n + 2)
    # indices whose probability mass is wide enough to separate from f32 rounding
    wide = np.nonzero(ref >= 1e-5)[0]
    picks = rng.choice(wide, size=min(len(wide), 8), replace=False)
    assert len(picks) > 0
    for i in picks:
        lo = c[i - 1] if i else 0.0
        r = float(0.5 * (lo + c[i]))          # midway inside the probability mass of index i
        ops.softmax_sample(tkdev, ld, probs, sampled, n, temperature, r)
        assert int(host(sampled)[0]) == oracle.sample_index(ref, r) == i
    p = host(probs)
    assert np.abs(p - ref).max() / ref.max() <= 1e-6


def test_sampler_rejects_bad_arguments(torch_cuda, tkdev):
    L = _lib.lib()
    t = torch_cuda.zeros(4, device="cuda")
    p = t.data_ptr()
    assert L.tk_argmax(tkdev.handle, p, 0, p) == _lib.TK_ERR_ARG
    assert L.tk_softmax_sample(tkdev.handle, p, p, p, 4, 0.0, 0.5) == _lib.TK_ERR_ARG
    assert L.tk_softmax_sample(tkdev.handle, None, p, p, 4, 1.0, 0.5) == _lib.TK_ERR_ARG
