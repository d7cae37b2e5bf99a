"""rw4_decode_attention (one decode step's attention over a bf16 static KV cache, the length read
on the device) against fp32 attention over the same bf16 cache, and replayed from a CUDA graph
as the position advances."""
import pytest
import torch

from rocketllm_b200 import _lib, kernels

pytestmark = pytest.mark.gpu


def reference(q, k, v, pos, scale):
    """fp32 softmax(scale q K^T) V over positions 0..pos, grouped-query heads."""
    b, h, d = q.shape
    kvh = k.shape[1]
    g = h // kvh
    kk = k[:, :, :pos + 1].float().repeat_interleave(g, dim=1)
    vv = v[:, :, :pos + 1].float().repeat_interleave(g, dim=1)
    s = torch.einsum("bhd,bhtd->bht", q.float(), kk) * scale
    return torch.einsum("bht,bhtd->bhd", s.softmax(-1), vv)


def run(q, k, v, pos_t, scale, out, stream=None):
    b, h, d = q.shape
    stream = stream or torch.cuda.current_stream().cuda_stream
    _lib.call("rw4_decode_attention", q.data_ptr(), b, h, k.shape[1], d, k.data_ptr(),
              v.data_ptr(), k.shape[2], pos_t.data_ptr(), scale, out.data_ptr(), stream)


@pytest.mark.parametrize("b,h,kvh,d,cap,pos", [
    (1, 32, 8, 128, 2176, 2047),     # Llama-3-8B shape, batch 1, 2K context
    (16, 32, 8, 128, 2176, 2100),    # batch 16
    (3, 8, 2, 64, 300, 250),         # head_dim 64, GQA 4
    (2, 8, 8, 128, 100, 0),          # the first position: one token
    (1, 32, 4, 64, 77, 76),          # GQA 8, the last position of a cache not a multiple of 64
    (4, 16, 16, 128, 4096, 4095),    # no grouping, full 4K cache
    (1, 12, 4, 128, 64, 63),         # GQA 3 (columns beyond G idle), one block
])
def test_decode_attention_matches_fp32(b, h, kvh, d, cap, pos):
    g = torch.Generator(device="cuda").manual_seed(b * 1000 + pos)
    q = torch.randn(b, h, d, generator=g, device="cuda").to(torch.bfloat16)
    k = torch.randn(b, kvh, cap, d, generator=g, device="cuda").to(torch.bfloat16)
    v = torch.randn(b, kvh, cap, d, generator=g, device="cuda").to(torch.bfloat16)
    # entries past the position must not matter: make them huge
    k[:, :, pos + 1:] = 3e4
    v[:, :, pos + 1:] = -3e4
    pos_t = torch.tensor([pos], dtype=torch.long, device="cuda")
    out = torch.empty(b, h, d, dtype=torch.bfloat16, device="cuda")
    scale = d ** -0.5
    run(q, k, v, pos_t, scale, out)
    torch.cuda.synchronize()
    assert kernels.device_status() == 0
    want = reference(q, k, v, pos, scale)
    err = float((out.float() - want).abs().max())
    # bf16 probabilities in the second product and the bf16 output: a few 1e-3 of |V| ~ 1
    assert err <= 1.5e-2, err
    # and against torch's own SDPA with the step's mask (what the fused step ran before)
    mask = torch.zeros(1, 1, 1, cap, device="cuda", dtype=torch.bfloat16)
    mask[..., pos + 1:] = float("-inf")
    sdpa = torch.nn.functional.scaled_dot_product_attention(
        q.view(b, h, 1, d), k, v, attn_mask=mask, scale=scale, enable_gqa=True).view(b, h, d)
    assert float((out.float() - sdpa.float()).abs().max()) <= 2e-2


def test_decode_attention_in_a_graph_follows_the_device_position():
    b, h, kvh, d, cap = 2, 32, 8, 128, 640
    g = torch.Generator(device="cuda").manual_seed(5)
    q = torch.randn(b, h, d, generator=g, device="cuda").to(torch.bfloat16)
    k = torch.randn(b, kvh, cap, d, generator=g, device="cuda").to(torch.bfloat16)
    v = torch.randn(b, kvh, cap, d, generator=g, device="cuda").to(torch.bfloat16)
    pos_t = torch.tensor([10], dtype=torch.long, device="cuda")
    out = torch.empty(b, h, d, dtype=torch.bfloat16, device="cuda")
    scale = d ** -0.5
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        run(q, k, v, pos_t, scale, out, side.cuda_stream)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        run(q, k, v, pos_t, scale, out)
    for p in (10, 63, 64, 65, 200, 639):
        pos_t.fill_(p)
        graph.replay()
        torch.cuda.synchronize()
        want = reference(q, k, v, p, scale)
        assert float((out.float() - want).abs().max()) <= 1.5e-2, p
        eager = torch.empty_like(out)
        run(q, k, v, pos_t, scale, eager)
        torch.cuda.synchronize()
        assert torch.equal(out, eager), p
    assert kernels.device_status() == 0


def test_decode_attention_rejects_what_it_does_not_cover():
    q = torch.zeros(1, 32, 96, dtype=torch.bfloat16, device="cuda")
    k = torch.zeros(1, 8, 64, 96, dtype=torch.bfloat16, device="cuda")
    pos_t = torch.zeros(1, dtype=torch.long, device="cuda")
    with pytest.raises(_lib.RW4Error):      # head_dim 96
        run(q, k, k, pos_t, 0.1, q)
    q = torch.zeros(1, 32, 128, dtype=torch.bfloat16, device="cuda")
    k = torch.zeros(1, 2, 64, 128, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(_lib.RW4Error):      # 16 query heads per kv head
        run(q, k, k, pos_t, 0.1, q)
