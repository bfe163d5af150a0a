"""SM-pair prefill GEMM (tcgen05.mma.cta_group::2) against an fp32 matmul of the same operands."""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _rand(*shape, std=1.0, seed=0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return (torch.randn(*shape, generator=g, device=DEV) * std).to(torch.bfloat16)


def _rel(x, y):
    return ((x.float() - y.float()).norm() / (y.float().norm() + 1e-6)).item()


@pytest.mark.parametrize("M,N,K", [(512, 1024, 4096), (256, 256, 64), (700, 800, 1000), (4096, 4096, 512),
                                   (300, 6144, 4096), (1, 32, 64)])
@pytest.mark.parametrize("tn", [0, 256, 128, 512])
def test_pair_gemm_store(M, N, K, tn):
    from mesh_b200 import ops
    a = _rand(M, K, seed=1)
    b = _rand(N, K, std=0.05, seed=2)
    out = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=DEV)
    ops.gemm_pair(a, b, out, tn=tn)
    torch.cuda.synchronize()
    ops.scratch(DEV).check("gemm_pair")
    want = a.float() @ b.float().T
    assert torch.isfinite(out.float()).all()
    assert _rel(out, want) < 1e-2, (M, N, K)


@pytest.mark.parametrize("M,I,K", [(512, 1792, 4096), (640, 128, 1024)])
@pytest.mark.parametrize("tn", [0, 512])
def test_pair_gemm_silu(M, I, K, tn):
    """Gate/up rows interleaved in 64-row blocks (the serving layout); out = SiLU(gate) * up."""
    from mesh_b200 import ops
    from mesh_b200.models.weights import interleave_gate_up
    a = _rand(M, K, seed=3)
    gate = _rand(I, K, std=0.05, seed=4)
    up = _rand(I, K, std=0.05, seed=5)
    w = interleave_gate_up(gate, up, I)
    out = torch.full((M, I), float("nan"), dtype=torch.bfloat16, device=DEV)
    ops.gemm_pair(a, w, out, ops.EPI_SILU_BF16, tn=tn)
    torch.cuda.synchronize()
    ops.scratch(DEV).check("gemm_pair silu")
    g = a.float() @ gate.float().T
    u = a.float() @ up.float().T
    want = torch.nn.functional.silu(g) * u
    assert _rel(out, want) < 2e-2


def test_pair_gemm_matches_one_sm_kernel():
    """The pair kernel and the one-SM kernel agree on a prefill-sized product."""
    from mesh_b200 import ops
    a = _rand(1024, 2048, seed=6)
    b = _rand(3072, 2048, std=0.05, seed=7)
    y_pair = ops.gemm_pair(a, b, torch.empty(1024, 3072, dtype=torch.bfloat16, device=DEV))
    y_one = ops.gemm(a, b, torch.empty_like(y_pair), ops.EPI_STORE_BF16, trans=False)
    torch.cuda.synchronize()
    assert _rel(y_pair, y_one) < 1e-2
