"""The triton_ops-named helpers (cache_ops) against their reference
semantics written in plain PyTorch (the reference's own CPU fallbacks,
triton_ops.py:107-346), on a B200.  Gathers and argmin exact; scatter
1e-6 relative (a mean in a different order); attention 1e-5 (fp32) /
1e-3 (fp16, bf16) normwise per row."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_gather_cache_kv(dtype):
    from infercache_b200.cache_ops import gather_cache_kv
    K = torch.randn(4, 300, 128, device="cuda").to(dtype)
    slots = torch.tensor([5, 0, 299, 17, 17, 100], device="cuda")
    got = gather_cache_kv(K, slots)
    assert torch.equal(got, K[:, slots, :].unsqueeze(0))
    Kv = torch.randn(300, 4, 128, device="cuda").to(dtype).transpose(0, 1)  # strided heads
    assert torch.equal(gather_cache_kv(Kv, slots), Kv[:, slots, :].unsqueeze(0))


@pytest.mark.parametrize("shape", [(3, 2, 1, 50), (3, 2, 50)])
def test_scatter_importance(shape):
    from infercache_b200.cache_ops import scatter_importance
    g = torch.Generator(device="cuda").manual_seed(1)
    w = torch.rand(shape, generator=g, device="cuda")
    slots = torch.randperm(64, generator=g, device="cuda")[:40]
    imp = torch.rand(64, generator=g, device="cuda")
    ref = imp.clone()
    agg = w.float().mean(dim=tuple(range(w.dim() - 1)))
    n = min(agg.shape[0], slots.shape[0])
    ref.scatter_add_(0, slots[:n], agg[:n])
    scatter_importance(w, slots, imp)
    assert torch.allclose(imp, ref, rtol=1e-6, atol=1e-7)


def test_topk_min_slot_first_index_and_nan():
    from infercache_b200.cache_ops import topk_min_slot
    x = torch.tensor([5.0, 1.0, 3.0, 1.0, 0.5, 0.5, 9.0], device="cuda")
    assert topk_min_slot(x, 1, 3) == 1
    assert topk_min_slot(x, 0, 7) == 4
    assert topk_min_slot(x, 3, 0) == 3
    y = torch.rand(5000, device="cuda")
    y[4321] = -1.0
    y[4400] = -1.0
    assert topk_min_slot(y, 100, 4800) == 4321
    y[200] = float("nan")
    assert topk_min_slot(y, 100, 4800) == int(100 + y[100:4900].cpu().argmin())


@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-5), (torch.float16, 1e-3), (torch.bfloat16, 1e-3)])
def test_compact_sdp_attention(dtype, tol):
    from infercache_b200.cache_ops import compact_sdp_attention
    H, budget, D, B = 4, 520, 128, 3
    g = torch.Generator(device="cuda").manual_seed(2)
    K = torch.randn(H, budget, D, generator=g, device="cuda").to(dtype)
    V = torch.randn(H, budget, D, generator=g, device="cuda").to(dtype)
    Q = torch.randn(B, H, 1, D, generator=g, device="cuda").to(dtype)
    slots = torch.randperm(budget, generator=g, device="cuda")[:333].sort().values
    got = compact_sdp_attention(Q, K, V, slots)
    Kc, Vc = K[:, slots].float(), V[:, slots].float()
    s = torch.einsum("bhd,hfd->bhf", Q[:, :, 0].float(), Kc) * D ** -0.5
    ref = torch.einsum("bhf,hfd->bhd", s.softmax(-1), Vc)
    err = ((got[:, :, 0].float() - ref).abs().amax(-1) / ref.abs().amax(-1)).max()
    assert float(err) < tol + (2 ** -8 if dtype == torch.bfloat16 else 2 ** -11 if dtype == torch.float16 else 0)


def test_importance_tracker():
    from infercache_b200.cache_ops import GPUImportanceTracker
    t = GPUImportanceTracker(32)
    cpu = torch.arange(32, dtype=torch.float32)
    t.sync_from_cpu(cpu)
    t.apply_decay(0.5)
    t.scatter_add(torch.tensor([3, 4], device="cuda"), torch.ones(1, 1, 1, 2, device="cuda"))
    out = torch.empty(32)
    t.sync_to_cpu(out)
    ref = cpu * 0.5
    ref[3] += 1
    ref[4] += 1
    assert torch.equal(out, ref)
    assert t.argmin_l2(10, 5) == 10
