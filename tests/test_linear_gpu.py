"""GPU parity of rw4_linear (dequant-GEMV and GEMM paths) with the oracle, through the C ABI.

Tolerance: the device output is bf16 of an fp32 accumulation, so each element may differ from the
fp32 oracle by one bf16 rounding (2^-8 relative) plus accumulation-order noise; the bound used is
|y - ref| <= ref_abs / 128 + 2e-3 * rms(ref).
"""
import numpy as np
import pytest
import torch

from oracle import rw4_oracle as o
from rocketllm_b200 import kernels
from rocketllm_b200.synthetic import make_activation, make_weight

pytestmark = pytest.mark.gpu


def check_close(y, ref):
    y = y.float().cpu().numpy()
    rms = float(np.sqrt(np.mean(ref.astype(np.float64) ** 2))) + 1e-12
    err = np.abs(y - ref)
    bound = np.abs(ref) / 128 + 2e-3 * rms
    assert np.all(err <= bound), f"max err {err.max():.4g}, worst excess {(err - bound).max():.4g}"


def oracle_linear(x, packed, scale, zero, rows=None, path=None):
    """The oracle over the weight the selected kernel multiplies by: the tensor-core GEMM uses the
    reference's bf16-rounded dequantized weight, the GEMV the exact fp32 weight."""
    xb = x.cpu().contiguous().view(torch.int16).numpy().view(np.uint16)
    p, s, z = packed.cpu().numpy(), scale.cpu().numpy(), zero.cpu().numpy()
    if rows is not None:
        p, s, z = p[rows], s[rows], z[rows]
    m, k = x.shape
    gemm = (path if path is not None else kernels.linear_path(m, k, packed.shape[0])) == 2
    return o.linear(xb, p, s, z, bf16_weight=gemm)


@pytest.mark.parametrize("m", [1, 2, 3, 4, 7, 8, 9, 15, 16, 17, 33, 64])
@pytest.mark.parametrize("k,n", [(4096, 512), (320, 136), (1024, 4104), (8192, 1024), (4096, 4096)])
def test_linear_matches_oracle(cuda, m, k, n):
    packed, scale, zero = make_weight(n, k, device=cuda, seed=m + k)
    x = make_activation(m, k, device=cuda, seed=n)
    y = kernels.linear(x, packed, scale, zero)
    torch.cuda.synchronize()
    check_close(y, oracle_linear(x, packed, scale, zero))


@pytest.mark.parametrize("k,n", [(32768, 512), (53248, 1024), (53248, 16384)])
def test_linear_long_k_one_row(cuda, k, n):
    """One activation row with a long K (converted in the GEMV, or by the x-prep pass when the CTA's
    K range passes 32 stages)."""
    packed, scale, zero = make_weight(n, k, device=cuda, seed=k + n)
    x = make_activation(1, k, device=cuda, seed=5)
    y = kernels.linear(x, packed, scale, zero)
    torch.cuda.synchronize()
    assert kernels.device_status() == 0
    rows = np.arange(0, n, max(1, n // 256))
    check_close(y[:, torch.from_numpy(rows).to(cuda)],
                oracle_linear(x, packed, scale, zero, rows=rows))


def test_linear_golden_reference_output(golden, cuda):
    """The reference's own bf16 F.linear over its dequantized weight (make_golden.py)."""
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    x = dev(golden["sweep.x"].view(np.int16)).view(torch.bfloat16)
    y = kernels.linear(x, dev(golden["sweep.packed"]), dev(golden["sweep.scale"]),
                       dev(golden["sweep.zero"]))
    check_close(y, golden["sweep.y_f32"])


@pytest.mark.parametrize("m", [17, 64, 255, 256, 300, 512])
@pytest.mark.parametrize("k,n", [(4096, 4096), (1024, 200)])
def test_gemm_matches_oracle(cuda, m, k, n):
    """The tcgen05 GEMM itself (forced with path=2, so the test holds whatever the dispatcher
    picks for these sizes), all three token-tile widths and ragged N."""
    packed, scale, zero = make_weight(n, k, device=cuda, seed=m + n)
    x = make_activation(m, k, device=cuda, seed=k + m)
    y = kernels.linear(x, packed, scale, zero, path=2)
    torch.cuda.synchronize()
    assert kernels.device_status() == 0
    check_close(y, oracle_linear(x, packed, scale, zero, path=2))


@pytest.mark.parametrize("k,n,m", [(16384, 53248, 1), (16384, 53248, 16), (8192, 28672, 1),
                                   (8192, 28672, 16), (16384, 53248, 2048), (4096, 14336, 512)])
def test_linear_full_size_sampled_rows(cuda, k, n, m):
    """Full sweep shapes: the oracle recomputes a seeded sample of output rows."""
    packed, scale, zero = make_weight(n, k, device=cuda, seed=7)
    x = make_activation(m, k, device=cuda, seed=8)
    y = kernels.linear(x, packed, scale, zero)
    rows = np.sort(np.random.default_rng(0).choice(n, 96, replace=False))
    rows = np.concatenate([rows, [0, n - 1]])
    ref = oracle_linear(x, packed, scale, zero, rows=rows)
    check_close(y[:, torch.from_numpy(rows).to(cuda)], ref)


def test_linear_is_linear_in_x(cuda):
    """Size-independent property: W(a x1 + x2) = a W x1 + W x2 within bf16 rounding."""
    packed, scale, zero = make_weight(14336, 4096, device=cuda, seed=3)
    x1 = make_activation(4, 4096, device=cuda, seed=4)
    y1 = kernels.linear(x1, packed, scale, zero).float()
    y2 = kernels.linear((2 * x1.float()).to(torch.bfloat16), packed, scale, zero).float()
    assert torch.allclose(y2, 2 * y1, rtol=1 / 64, atol=1e-2)


@pytest.mark.parametrize("sigma", [1e-4, 1e-3, 1e-2, 1.0, 100.0])
@pytest.mark.parametrize("m", [1, 3, 16])
@pytest.mark.parametrize("k,n", [(4096, 1024), (16384, 512)])
def test_linear_any_activation_scale(cuda, sigma, m, k, n):
    """x ~ N(0, sigma^2) over six decades, plus one row whose channels 7, 700 and 3000 are outliers
    (10^3 to 10^4 times sigma): within the bf16 tolerance of the oracle at every scale."""
    packed, scale, zero = make_weight(n, k, device=cuda, seed=11)
    x = make_activation(m, k, device=cuda, seed=12).float() * sigma
    x[0, [7, 700, 3000]] = torch.tensor([1e3, -4e3, 1e4], device=cuda) * sigma
    x = x.to(torch.bfloat16)
    y = kernels.linear(x, packed, scale, zero)
    torch.cuda.synchronize()
    check_close(y, oracle_linear(x, packed, scale, zero))


@pytest.mark.parametrize("m", [1, 5, 16, 40])
def test_linear_power_of_two_scaling_is_exact(cuda, m):
    """y(2^j x) = 2^j y(x) bit for bit: each row's fp16 conversion follows its own exponent."""
    packed, scale, zero = make_weight(4096, 8192, device=cuda, seed=13)
    x = make_activation(m, 8192, device=cuda, seed=14)
    y = kernels.linear(x, packed, scale, zero)
    for j in (-40, -12, -1, 3, 20):
        ys = kernels.linear((x.float() * 2.0 ** j).to(torch.bfloat16), packed, scale, zero)
        assert torch.equal(ys.float(), y.float() * 2.0 ** j), f"2^{j}"


@pytest.mark.parametrize("k,n", [(4096, 4096), (14336, 4096), (4096, 14336), (53248, 1024)])
def test_linear_row_independent_of_batch(cuda, k, n):
    """A row's output has the same bits alone (M = 1), in a decode batch and in the 16-row slices of
    a larger M (up to the GEMV's 64 rows): decode batches and speculative verify passes round
    exactly like one-token steps.  (53248 x 1024: a one-row launch long enough to go through the
    x-prep pass as well.)"""
    packed, scale, zero = make_weight(n, k, device=cuda, seed=15)
    x = make_activation(64, k, device=cuda, seed=16)
    x[5] *= 1e-3  # rows of very different magnitude side by side
    x[9] *= 300
    alone = torch.cat([kernels.linear(x[i:i + 1], packed, scale, zero) for i in range(64)])
    for m in (2, 4, 8, 9, 16, 17, 33, 64):
        # past 16 rows the GEMV runs in 16-row slices (path 3; the default there may be the
        # tcgen05 decode GEMM, tested below)
        y = kernels.linear(x[:m], packed, scale, zero, path=1 if m <= 16 else 3)
        assert torch.equal(y, alone[:m]), f"M={m}"
    torch.cuda.synchronize()
    check_close(alone, oracle_linear(x, packed, scale, zero))


@pytest.mark.parametrize("k,n", [(4096, 14336), (1024, 12288), (14336, 12416)])
@pytest.mark.parametrize("m", [17, 24, 32, 33, 48, 64])
def test_decode_gemm_matches_oracle(cuda, m, k, n):
    """The tcgen05 decode GEMM (path 4, forced here for 17-64 rows; the library picks it for 49-64):
    exact fp32 weights through fp16 code patterns and per-group scales applied from TMEM, against
    the oracle's exact-weight linear; rows of very different magnitude side by side."""
    assert kernels.linear_path(m, k, n) == (4 if m >= 49 else 3)
    packed, scale, zero = make_weight(n, k, device=cuda, seed=m + 3 * k)
    x = make_activation(m, k, device=cuda, seed=n + m)
    x[1] *= 1e-3
    x[m - 1] *= 300
    y = kernels.linear(x, packed, scale, zero, path=4)
    torch.cuda.synchronize()
    assert kernels.device_status() == 0
    rows = np.arange(0, n, max(1, n // 512))
    check_close(y[:, torch.from_numpy(rows).to(cuda)],
                oracle_linear(x, packed, scale, zero, rows=rows, path=4))


@pytest.mark.parametrize("k,n", [(4096, 14336), (14336, 12416)])
def test_decode_gemm_rows_independent_of_batch(cuda, k, n):
    """A row's output from the decode GEMM has the same bits at every M of one column tile
    (17-32, 33-64), and a power-of-two scaling of x scales y exactly."""
    packed, scale, zero = make_weight(n, k, device=cuda, seed=21)
    x = make_activation(64, k, device=cuda, seed=22)
    x[3] *= 1e-3
    x[20] *= 300
    y32 = kernels.linear(x[:32], packed, scale, zero, path=4)
    for m in (17, 24, 31):
        assert torch.equal(kernels.linear(x[:m], packed, scale, zero, path=4), y32[:m]), f"M={m}"
    y64 = kernels.linear(x, packed, scale, zero, path=4)
    for m in (33, 48, 63):
        assert torch.equal(kernels.linear(x[:m], packed, scale, zero, path=4), y64[:m]), f"M={m}"
    for j in (-20, 7):
        ys = kernels.linear((x.float() * 2.0 ** j).to(torch.bfloat16), packed, scale, zero,
                            path=4)
        assert torch.equal(ys.float(), y64.float() * 2.0 ** j), f"2^{j}"
    assert kernels.device_status() == 0


@pytest.mark.parametrize("m,k,n", [(1, 4096, 4096), (5, 4096, 6144), (40, 1024, 2048),
                                   (56, 4096, 12288)])
def test_linear_residual_epilogue(cuda, m, k, n):
    """rw4_linear_residual_ws (a decoder layer's o_proj / down_proj with its residual add): the
    GEMV's epilogue (one row, a decode batch), the 16-row slices, and the tcgen05 decode GEMM's
    epilogue (56 rows) all give bf16(residual + bf16(x . W^T)) -- the module's two roundings --
    bit for bit, also in place (the residual is the output buffer)."""
    from rocketllm_b200 import _lib
    w = make_weight(n, k, device=cuda, seed=31)
    x = make_activation(m, k, device=cuda, seed=32)
    res = make_activation(m, n, device=cuda, seed=33)
    want = (kernels.linear(x, *w).float() + res.float()).to(torch.bfloat16)
    wsb = kernels.linear_workspace_bytes(m, k, n)
    ws = torch.empty(max(wsb, 256), dtype=torch.uint8, device=cuda)
    stream = torch.cuda.current_stream(cuda).cuda_stream
    for in_place in (False, True):
        y = res.clone() if in_place else torch.empty(m, n, dtype=torch.bfloat16, device=cuda)
        _lib.call("rw4_linear_residual_ws", x.data_ptr(), m, k, w[0].data_ptr(), w[1].data_ptr(),
                  w[2].data_ptr(), n, 64, y.data_ptr() if in_place else res.data_ptr(),
                  y.data_ptr(), ws.data_ptr(), ws.numel(), stream)
        torch.cuda.synchronize()
        assert torch.equal(y, want), f"in_place={in_place}"
    assert kernels.device_status() == 0


@pytest.mark.parametrize("m,k,n", [(1, 4096, 6144), (1, 4096, 1024), (1, 14336, 4096),
                                   (1, 4096, 28672), (1, 17408, 12288), (2, 4096, 6144),
                                   (16, 2048, 11264), (40, 4096, 4096), (56, 4096, 12288),
                                   (3, 1600, 1024), (1, 1600, 1024)])
def test_linear_rmsnorm_matches_norm_then_linear(cuda, m, k, n):
    """rw4_linear_rmsnorm_ws (a layer norm folded into the projection's activation conversion)
    gives the bits of rw4_rmsnorm followed by the projection: the same rounding sequence and the
    same summation order for the row's mean square.  One row: the GEMV's own prologue normalises
    (4096 x 1024 splits K over 4 CTAs, each normalising the whole row for its maximum); 17408 x
    12288: 34 KB of row in one CTA, beyond the prologue's 32 KB, so through the x-prep pass.  (1600: K % 512 != 0, normalised
    first.)"""
    import ctypes
    from rocketllm_b200 import _lib
    w = make_weight(n, k, device=cuda, seed=41)
    x = make_activation(m, k, device=cuda, seed=42) * 3
    nw = (1 + 0.1 * make_activation(1, k, device=cuda, seed=43)).to(torch.bfloat16).view(k)
    stream = torch.cuda.current_stream(cuda).cuda_stream
    xn = torch.empty_like(x)
    _lib.call("rw4_rmsnorm", x.data_ptr(), nw.data_ptr(), m, k, 1e-5, xn.data_ptr(), stream)
    want = kernels.linear(xn, *w)
    nb = ctypes.c_size_t(0)
    _lib.call("rw4_linear_rmsnorm_workspace_size", m, k, n, ctypes.byref(nb))
    ws = torch.empty(max(nb.value, 256), dtype=torch.uint8, device=cuda)
    y = torch.empty(m, n, dtype=torch.bfloat16, device=cuda)
    _lib.call("rw4_linear_rmsnorm_ws", x.data_ptr(), m, k, nw.data_ptr(), 1e-5, w[0].data_ptr(),
              w[1].data_ptr(), w[2].data_ptr(), n, 64, y.data_ptr(), ws.data_ptr(), ws.numel(),
              stream)
    torch.cuda.synchronize()
    assert kernels.device_status() == 0
    assert torch.equal(y, want)


@pytest.mark.parametrize("m,k,n", [(1, 4096, 28672), (1, 2048, 11264), (2, 4096, 28672),
                                   (9, 4096, 28672), (16, 2048, 11264), (40, 4096, 28672),
                                   (56, 4096, 28672), (1, 4096, 2048), (3, 1600, 2048),
                                   (1, 17408, 12288)])
def test_linear_rmsnorm_swiglu_matches_three_calls(cuda, m, k, n):
    """rw4_linear_rmsnorm_swiglu_ws over a [gate; up] weight gives the bits of
    rw4_linear_rmsnorm_ws followed by rw4_silu_mul: one launch where the GEMV's shape pairs gate
    and up rows (64-, 32- and 16-row shapes; one row in the GEMV's prologue, a batch through the
    x-prep pass), the two calls otherwise (4096 x 2048 splits K; 56 rows take the decode GEMM;
    K % 512 != 0)."""
    import ctypes
    from rocketllm_b200 import _lib
    w = make_weight(n, k, device=cuda, seed=51)
    x = make_activation(m, k, device=cuda, seed=52) * 3
    nw = (1 + 0.1 * make_activation(1, k, device=cuda, seed=53)).to(torch.bfloat16).view(k)
    stream = torch.cuda.current_stream(cuda).cuda_stream
    nb = ctypes.c_size_t(0)
    _lib.call("rw4_linear_rmsnorm_workspace_size", m, k, n, ctypes.byref(nb))
    ws = torch.empty(max(nb.value, 256), dtype=torch.uint8, device=cuda)
    gu = torch.empty(m, n, dtype=torch.bfloat16, device=cuda)
    _lib.call("rw4_linear_rmsnorm_ws", x.data_ptr(), m, k, nw.data_ptr(), 1e-5, w[0].data_ptr(),
              w[1].data_ptr(), w[2].data_ptr(), n, 64, gu.data_ptr(), ws.data_ptr(), ws.numel(),
              stream)
    want = torch.empty(m, n // 2, dtype=torch.bfloat16, device=cuda)
    _lib.call("rw4_silu_mul", gu.data_ptr(), m, n // 2, want.data_ptr(), stream)
    _lib.call("rw4_linear_rmsnorm_swiglu_workspace_size", m, k, n, ctypes.byref(nb))
    ws2 = torch.empty(max(nb.value, 256), dtype=torch.uint8, device=cuda)
    y = torch.full((m, n // 2), float("nan"), dtype=torch.bfloat16, device=cuda)
    _lib.call("rw4_linear_rmsnorm_swiglu_ws", x.data_ptr(), m, k, nw.data_ptr(), 1e-5,
              w[0].data_ptr(), w[1].data_ptr(), w[2].data_ptr(), n, 64, y.data_ptr(),
              ws2.data_ptr(), ws2.numel(), stream)
    torch.cuda.synchronize()
    assert kernels.device_status() == 0
    assert torch.equal(y, want)
    # and the model's own act_fn(gate) * up over those gate / up values
    g, u = gu[:, :n // 2].float(), gu[:, n // 2:].float()
    ref = (torch.nn.functional.silu(g).to(torch.bfloat16).float() * u).to(torch.bfloat16)
    assert (y.float() - ref.float()).abs().max().item() <= 1e-2 * ref.float().abs().max().item()


def test_linear_deterministic(cuda):
    packed, scale, zero = make_weight(4096, 14336, device=cuda, seed=5)
    x = make_activation(16, 14336, device=cuda, seed=6)
    a = kernels.linear(x, packed, scale, zero)
    b = kernels.linear(x, packed, scale, zero)
    assert torch.equal(a, b)


@pytest.mark.parametrize("k,n", [(4096, 6144), (4096, 14336), (14336, 4096)])
@pytest.mark.parametrize("m", [1, 8, 32, 127, 128])
def test_linear_repeats_bit_for_bit(cuda, k, n, m):
    """Forty launches on the same inputs, each compared (a host sync between launches) with the
    first: every path's ring protocol must leave no room for a slot being refilled while its last
    reader is still on it.  Shapes with fewer weight tiles than SMs at M = 127-128 (one token tile
    on the tcgen05 GEMM) are where a missing proxy fence between the consumers' generic reads of
    a codes slot and its TMA refill showed as run-to-run differences in a prefill."""
    w = make_weight(n, k, device=cuda, seed=11)
    x = make_activation(m, k, device=cuda, seed=12)
    first = kernels.linear(x, *w)
    diffs = sum(int(not torch.equal(first, kernels.linear(x, *w))) for _ in range(40))
    assert kernels.device_status() == 0
    assert diffs == 0, f"{diffs} of 40 launches differ from the first"
