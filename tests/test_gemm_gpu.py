"""tcgen05 GEMM numerics against an fp32 PyTorch reference of the same op."""
import pytest
import torch

from flare_b200.ops.gemm import gemm, gemm_reference

pytestmark = pytest.mark.gpu


def _rand(rows, cols, device):
    """bf16 [rows, cols] view whose row pitch is padded to a multiple of 8 elements."""
    ld = (cols + 7) // 8 * 8
    full = (torch.randn(rows, ld, device=device) * 0.5).to(torch.bfloat16)
    return full[:, :cols]


@pytest.mark.parametrize("a_t,b_t", [(False, False), (False, True), (True, False), (True, True)])
@pytest.mark.parametrize("M,N,K", [(128, 128, 64), (256, 192, 320), (300, 100, 200), (1024, 512, 1024)])
def test_gemm_majors(cuda, a_t, b_t, M, N, K):
    torch.manual_seed(0)
    a = _rand(K, M, device=cuda) if a_t else _rand(M, K, device=cuda)
    b = _rand(K, N, device=cuda) if b_t else _rand(N, K, device=cuda)
    # pad leading dims to multiples of 8 as the kernels require 16-byte row pitch
    out = torch.zeros(M, (N + 7) // 8 * 8, dtype=torch.float32, device=cuda)[:, :N]
    gemm(a, b, a_t=a_t, b_t=b_t, out=out)
    ref = gemm_reference(a, b, a_t=a_t, b_t=b_t)
    torch.cuda.synchronize()
    err = (out - ref).abs().max().item()
    scale = ref.abs().max().item()
    assert err <= 2e-3 * scale + 1e-3, (err, scale)


@pytest.mark.parametrize("bn", [64, 128, 256])
def test_gemm_tile_widths_bf16_out(cuda, bn):
    torch.manual_seed(1)
    M, N, K = 512, 512, 256
    a, b = _rand(M, K, device=cuda), _rand(N, K, device=cuda)
    bias = (torch.randn(N, device=cuda) * 0.1).to(torch.bfloat16)
    out = gemm(a, b, bias=bias, relu=True, bn=bn)
    ref = gemm_reference(a, b, bias=bias, relu=True)
    torch.testing.assert_close(out.float(), ref, rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("bn", [64, 128, 256])
def test_gemm_bf16_out_tails_strided_and_unaligned_bias(cuda, bn):
    # row and column tails (a partial last 32-column chunk), an output wider than N, and a bias that
    # starts one element into its buffer (not 16-byte aligned)
    torch.manual_seed(4)
    M, N, K = 300, 200, 320
    a, b = _rand(M, K, device=cuda), _rand(N, K, device=cuda)
    bias = (torch.randn(N + 1, device=cuda) * 0.1).to(torch.bfloat16)[1:]
    out = torch.full((M, 216), 7.0, dtype=torch.bfloat16, device=cuda)
    gemm(a, b, bias=bias, relu=True, out=out[:, :N], bn=bn)
    ref = gemm_reference(a, b, bias=bias, relu=True)
    torch.testing.assert_close(out[:, :N].float(), ref, rtol=2e-2, atol=2e-2)
    assert bool((out[:, N:] == 7.0).all())  # nothing written past N
    mask = _rand(M, N, device=cuda)
    colsum = torch.zeros(N, device=cuda)
    got = gemm(a, b, mask=mask, colsum=colsum, bn=bn)
    want = gemm_reference(a, b, mask=mask)
    torch.testing.assert_close(got.float(), want, rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(colsum, want.sum(0), rtol=1e-2, atol=5e-2)


def test_gemm_epilogue_mask_colsum_accumulate(cuda):
    torch.manual_seed(2)
    M, N, K = 384, 256, 192
    a, b = _rand(M, K, device=cuda), _rand(K, N, device=cuda)
    mask = _rand(M, N, device=cuda)
    colsum = torch.zeros(N, device=cuda)
    out = gemm(a, b, b_t=True, mask=mask, colsum=colsum)
    ref = gemm_reference(a, b, b_t=True, mask=mask)
    torch.testing.assert_close(out.float(), ref, rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(colsum, ref.sum(0), rtol=1e-2, atol=5e-2)
    acc = torch.ones(M, N, device=cuda)
    gemm(a, b, b_t=True, out=acc, accumulate=True, alpha=0.5)
    torch.testing.assert_close(acc, 1 + 0.5 * gemm_reference(a, b, b_t=True), rtol=2e-3, atol=2e-3)


def test_gemm_small_k_padded_input(cuda):
    # bottom-MLP first layer: K = 16 (13 features padded)
    torch.manual_seed(3)
    x = _rand(1024, 16, device=cuda)
    w = _rand(512, 16, device=cuda)
    out = gemm(x, w, out_dtype=torch.float32)
    torch.testing.assert_close(out, gemm_reference(x, w), rtol=2e-3, atol=2e-3)


@pytest.mark.parametrize("M,N,K", [(512, 480, 8192), (128, 16, 4096), (1024, 1024, 2048)])
def test_gemm_split_k_weight_gradient(cuda, M, N, K):
    """dW = dY^T X with K = batch: both operands MN-major, fp32 accumulate -> split-K path."""
    torch.manual_seed(5)
    dy = _rand(K, M, device=cuda)
    x = _rand(K, N, device=cuda)
    out = torch.full((M, N), 0.25, device=cuda)
    gemm(dy, x, a_t=True, b_t=True, out=out, accumulate=True)
    ref = 0.25 + gemm_reference(dy, x, a_t=True, b_t=True)
    torch.testing.assert_close(out, ref, rtol=2e-3, atol=2e-2)


@pytest.mark.parametrize("a_t,b_t", [(False, False), (False, True), (True, False), (True, True)])
@pytest.mark.parametrize("M,N,K", [(256, 256, 64), (512, 384, 320), (300, 200, 200), (1024, 1024, 1024),
                                   (8192, 128, 256)])
def test_gemm_cta_pair_majors(cuda, a_t, b_t, M, N, K):
    """CTA-pair tiles (cta_group::2, 256 rows over two SMs): every operand major, row / column / K tails
    (300 rows leave the second pair's odd CTA with no valid row)."""
    torch.manual_seed(10)
    a = _rand(K, M, device=cuda) if a_t else _rand(M, K, device=cuda)
    b = _rand(K, N, device=cuda) if b_t else _rand(N, K, device=cuda)
    out = torch.zeros(M, (N + 7) // 8 * 8, dtype=torch.float32, device=cuda)[:, :N]
    gemm(a, b, a_t=a_t, b_t=b_t, out=out, pair=True)
    ref = gemm_reference(a, b, a_t=a_t, b_t=b_t)
    torch.cuda.synchronize()
    err = (out - ref).abs().max().item()
    scale = ref.abs().max().item()
    assert err <= 2e-3 * scale + 1e-3, (err, scale)


@pytest.mark.parametrize("bn", [128, 256])
def test_gemm_cta_pair_epilogues(cuda, bn):
    """Pair tiles with the MLP epilogues: bias + ReLU (bf16 out), ReLU-backward mask + column sums,
    fp32 accumulate, and split-K weight gradients (both operands MN-major)."""
    torch.manual_seed(11)
    M, N, K = 768, 512, 448
    a, b = _rand(M, K, device=cuda), _rand(N, K, device=cuda)
    bias = (torch.randn(N, device=cuda) * 0.1).to(torch.bfloat16)
    out = gemm(a, b, bias=bias, relu=True, bn=bn, pair=True)
    torch.testing.assert_close(out.float(), gemm_reference(a, b, bias=bias, relu=True), rtol=2e-2, atol=2e-2)
    mask = _rand(M, N, device=cuda)
    colsum = torch.zeros(N, device=cuda)
    out = gemm(a, b, mask=mask, colsum=colsum, bn=bn, pair=True)
    ref = gemm_reference(a, b, mask=mask)
    torch.testing.assert_close(out.float(), ref, rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(colsum, ref.sum(0), rtol=1e-2, atol=5e-2)
    acc = torch.ones(M, N, device=cuda)
    gemm(a, b, out=acc, accumulate=True, alpha=0.5, bn=bn, pair=True)
    torch.testing.assert_close(acc, 1 + 0.5 * gemm_reference(a, b), rtol=2e-3, atol=2e-3)
    dy, x = _rand(8192, 512, device=cuda), _rand(8192, 256, device=cuda)
    dw = torch.full((512, 256), 0.25, device=cuda)
    gemm(dy, x, a_t=True, b_t=True, out=dw, accumulate=True, bn=bn, pair=True)
    torch.testing.assert_close(dw, 0.25 + gemm_reference(dy, x, a_t=True, b_t=True), rtol=2e-3, atol=2e-2)
