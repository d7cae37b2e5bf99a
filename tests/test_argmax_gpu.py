"""rw4_argmax_rows (the fused decode step's greedy choice) against torch.argmax on the same bf16
scores: random rows at the vocabularies of the benchmark models, ties, NaN, -inf, a strided view,
a vocabulary that is not a whole number of 16-byte vectors, and one smaller than the cluster."""
import pytest
import torch

from rocketllm_b200 import _lib, kernels

pytestmark = pytest.mark.gpu


def check(scores):
    got = kernels.argmax_rows(scores)
    torch.cuda.synchronize()
    want = scores.argmax(-1, keepdim=True)
    assert torch.equal(got, want), (got.flatten()[:8].tolist(), want.flatten()[:8].tolist())


@pytest.mark.parametrize("rows,v", [(1, 128256), (16, 128256), (32, 32000), (3, 32001), (2, 5),
                                    (4, 8), (1, 1)])
def test_argmax_matches_torch(rows, v):
    g = torch.Generator(device="cuda").manual_seed(rows * 7 + v)
    check(torch.randn(rows, v, generator=g, device="cuda").to(torch.bfloat16))


def test_argmax_ties_take_the_first_index():
    s = torch.zeros(4, 128256, dtype=torch.bfloat16, device="cuda")
    s[0, [5, 70000, 128255]] = 3.0           # first of three equal maxima
    s[1, [128255, 100000]] = 2.5             # maxima in two CTAs' shares
    s[2] = -1.0                              # a constant row: index 0
    s[3, 16031:16034] = 1.0                  # across the first two CTAs' boundary
    check(s)
    # bf16 rounding makes many near values equal: heavy ties everywhere
    g = torch.Generator(device="cuda").manual_seed(3)
    check((torch.rand(8, 32000, generator=g, device="cuda") * 4).round().to(torch.bfloat16))


def test_argmax_nan_and_infinities():
    s = torch.randn(5, 32000, device="cuda").to(torch.bfloat16)
    s[0, 123] = float("nan")
    s[0, 31000] = float("nan")
    s[1, 4000] = float("inf")
    s[1, 20000] = float("nan")
    s[2] = float("-inf")
    s[3, 7] = float("inf")
    s[3, 6] = float("inf")
    s[4, 31999] = float("nan")
    check(s)


def test_argmax_on_a_strided_view_and_into_a_buffer():
    wide = torch.randn(6, 32768, device="cuda").to(torch.bfloat16)
    view = wide[:, :32000]                   # row stride 32768, V 32000
    check(view)
    odd = torch.randn(3, 32007, device="cuda").to(torch.bfloat16)[:, 3:32003]  # unaligned start
    check(odd)
    out = torch.full((6, 1), -5, dtype=torch.int64, device="cuda")
    kernels.argmax_rows(view, out=out)
    torch.cuda.synchronize()
    assert torch.equal(out, view.argmax(-1, keepdim=True))


def test_argmax_rejects_bad_arguments():
    with pytest.raises(RuntimeError):
        _lib.call("rw4_argmax_rows", 0, 1, 10, 10, 0, None)          # null pointers
    x = torch.zeros(2, 10, dtype=torch.bfloat16, device="cuda")
    out = torch.zeros(2, 1, dtype=torch.int64, device="cuda")
    with pytest.raises(RuntimeError):
        _lib.call("rw4_argmax_rows", x.data_ptr(), 2, 10, 9, out.data_ptr(), None)  # ld < V
    with pytest.raises(RuntimeError):
        _lib.call("rw4_argmax_rows", x.data_ptr(), 2, 0, 10, out.data_ptr(), None)  # V = 0
    _lib.call("rw4_argmax_rows", x.data_ptr(), 0, 10, 10, out.data_ptr(), None)     # no rows
