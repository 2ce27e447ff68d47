"""This library's kernels against the reference's own CUDA kernels (foidfinder/backends/cuda/csrc/kernels.cu,
compiled for sm_100 by oracle/build_ref.py into oracle/_ref/) on the same inputs, at the PixAI shapes the
reference's kernels are written for (1024-wide rotations, the 4736-wide GELU hidden, 576/5184-token
attention). A second checker next to the CPU oracle; `test_reference_kernel_speed` also prints both
sides' timings (CUDA events, same stream) as a GPU speed bar.
"""

import math
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

LIB = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "pixai_kernels.so"
Q_SCALE = 0.125 * math.log2(math.e)  # engine.py:26


@pytest.fixture(scope="module")
def ref(cuda_device):
    if not LIB.is_file():
        pytest.skip("reference kernels not built (python -m oracle.build_ref)")
    torch.ops.load_library(str(LIB))
    return torch.ops.foidfinder


def _act(rows, cols, seed, d):
    g = torch.Generator(device=d).manual_seed(seed)
    x = torch.randn(rows, cols, generator=g, device=d)
    return torch.where(torch.rand(rows, cols, generator=g, device=d) < 0.01, x * 20, x).half()


def _codes_close(got, want, what):
    diff = (got.int() - want.int()).abs()
    assert diff.max().item() <= 1, f"{what}: code off by {diff.max().item()}"
    assert diff.float().mean().item() < 1e-3, f"{what}: {diff.float().mean().item():.2e} of codes differ"


@pytest.mark.parametrize("norm", [True, False])
def test_rot_q8_1024_matches_reference_kernel(ref, cuda_device, no_device_error, norm):
    from foidfinder_b200 import ops

    d, T = cuda_device, 2 * 5184
    x = _act(T, 1024, 1, d)
    g = torch.Generator(device=d).manual_seed(2)
    gamma = (1 + 0.1 * torch.randn(1024, generator=g, device=d)) if norm else None
    beta = (0.1 * torch.randn(1024, generator=g, device=d)) if norm else None
    q_ref, s_ref = torch.empty(T, 1024, dtype=torch.int8, device=d), torch.empty(T, device=d)
    q_got, s_got = torch.empty_like(q_ref), torch.empty_like(s_ref)
    ref.rot_q8_1024(x, gamma, beta, q_ref, s_ref)
    ops.rot_q8_1024(x, gamma, beta, q_got, s_got)
    torch.cuda.synchronize()
    torch.testing.assert_close(s_got, s_ref, rtol=2e-5, atol=0)
    _codes_close(q_got, q_ref, "rot_q8_1024")


def test_rot_q8_h128_matches_reference_kernel(ref, cuda_device, no_device_error):
    from foidfinder_b200 import ops

    d, T, C = cuda_device, 2 * 5184, 4736
    x = _act(T, C, 3, d)
    q_ref, s_ref = torch.empty(T, C, dtype=torch.int8, device=d), torch.empty(T, device=d)
    q_got, s_got = torch.empty_like(q_ref), torch.empty_like(s_ref)
    ref.rot_q8_h128(x, q_ref, s_ref)
    ops.rot_q8_h128(x, q_got, s_got)
    torch.cuda.synchronize()
    torch.testing.assert_close(s_got, s_ref, rtol=2e-5, atol=0)
    _codes_close(q_got, q_ref, "rot_q8_h128")


def _gemm_case(M, N, K, seed, d):
    g = torch.Generator(device=d).manual_seed(seed)
    A = torch.randint(-127, 128, (M, K), generator=g, device=d, dtype=torch.int8)
    W = torch.randint(-127, 128, (N, K), generator=g, device=d, dtype=torch.int8)
    rs = torch.rand(M, generator=g, device=d) * 0.05 / math.sqrt(K / 1024) + 1e-3
    cs = torch.rand(N, generator=g, device=d) * 1e-3 + 1e-5
    b = torch.randn(N, generator=g, device=d) * 0.1
    return A, W, rs, cs, b


@pytest.mark.parametrize(("N", "K"), [(1024, 1024), (1024, 4736)])
def test_gemm_residual_matches_reference_kernel(ref, cuda_device, no_device_error, N, K):
    from foidfinder_b200 import ops

    d, M = cuda_device, 2 * 5184
    A, W, rs, cs, b = _gemm_case(M, N, K, N + K, d)
    x0 = _act(M, N, 5, d)
    x_ref, x_got = x0.clone(), x0.clone()
    ref.gemm_s8(A, W, rs, cs, b, x_ref, 1, 3, None, None, 1.0)
    ops.gemm_s8(A, W, rs, cs, b, x_got, ops.EPI_RESIDUAL)
    torch.cuda.synchronize()
    torch.testing.assert_close(x_got.float(), x_ref.float(), atol=2e-3, rtol=2e-3)
    assert (x_got == x_ref).float().mean().item() > 0.999  # same fp16 staging + add, f32 rounding aside


def test_gemm_gelu_matches_reference_kernel(ref, cuda_device, no_device_error):
    from foidfinder_b200 import ops

    d, M, N, K = cuda_device, 2 * 5184, 4736, 1024
    A, W, rs, cs, b = _gemm_case(M, N, K, 7, d)
    h_ref = torch.empty(M, N, dtype=torch.float16, device=d)
    h_got = torch.empty_like(h_ref)
    ref.gemm_s8(A, W, rs, cs, b, h_ref, 2, 3, None, None, 1.0)
    ops.gemm_s8(A, W, rs, cs, b, h_got, ops.EPI_GELU)
    torch.cuda.synchronize()
    torch.testing.assert_close(h_got.float(), h_ref.float(), atol=2e-3, rtol=2e-3)


@pytest.mark.parametrize("seq", [576, 5184])
def test_gemm_qkv_rope_matches_reference_kernel(ref, cuda_device, no_device_error, seq):
    """The reference multiplies q by q_scale after RoPE (gemm.cuh:141-149); this library folds the attention
    scale into W, so its q columns are compared after the same multiplication."""
    from foidfinder_b200 import ops
    from foidfinder_b200.weights import axial_rope, window_order

    d, M, N, K = cuda_device, 2 * 5184, 3072, 1024
    A, W, rs, cs, b = _gemm_case(M, N, K, seq, d)
    if seq == 576:
        cos, sin = axial_rope(24, 1.0)
    else:
        cos, sin = axial_rope(72, 24 / 72)
        perm = window_order(72, 24)
        cos, sin = cos[perm], sin[perm]
    cos, sin = cos.contiguous().to(d), sin.contiguous().to(d)
    o_ref = torch.empty(M, N, dtype=torch.float16, device=d)
    o_got = torch.empty_like(o_ref)
    ref.gemm_s8(A, W, rs, cs, b, o_ref, 0, 3, cos, sin, Q_SCALE)
    ops.gemm_s8(A, W, rs, cs, b, o_got, ops.EPI_QKV_ROPE, rope_cos=cos.t().contiguous(), rope_sin=sin.t().contiguous(),
                rope_cols=2048, tokens=seq)
    torch.cuda.synchronize()
    got = o_got.float()
    got[:, :1024] *= Q_SCALE
    torch.testing.assert_close(got, o_ref.float(), atol=3e-3, rtol=3e-3)


@pytest.mark.parametrize(("seqs", "seq"), [(18, 576), (2, 5184)])
def test_attention_matches_reference_kernel(ref, cuda_device, no_device_error, seqs, seq):
    """The reference's attention computes softmax base 2 of q.k (q carries log2 e, engine.py:26); this
    library's with scale = ln 2 computes the same."""
    from foidfinder_b200 import ops

    d = cuda_device
    qkv = (_act(seqs * seq, 3072, 11, d).float() * 0.5).half()
    qkv[:, :1024] = (qkv[:, :1024].float() * Q_SCALE).half()
    o_ref = torch.empty(seqs * seq, 1024, dtype=torch.float16, device=d)
    o_got = torch.empty_like(o_ref)
    ref.attention(qkv, o_ref, seq)
    ops.attention(qkv, o_got, seq, 16, scale=math.log(2.0))
    torch.cuda.synchronize()
    # exact softmax base 2 in f64 (1% of the inputs are x20 outliers, so some rows are very peaked)
    q, k, v = qkv.double().view(seqs, seq, 3, 16, 64).permute(2, 0, 3, 1, 4)
    exact = (torch.softmax((q @ k.transpose(-1, -2)) * math.log(2.0), -1) @ v).transpose(1, 2).reshape(seqs * seq, 1024)
    err_got = (o_got.double() - exact).abs()
    err_ref = (o_ref.double() - exact).abs()
    print(f"\nattention {seqs}x{seq}: max |err| ours {err_got.max().item():.3e} reference kernel "
          f"{err_ref.max().item():.3e}; mean ours {err_got.mean().item():.3e} reference {err_ref.mean().item():.3e}")
    torch.testing.assert_close(o_got.double(), exact, atol=3e-3, rtol=1e-2)
    assert err_got.mean().item() <= 1.5 * err_ref.mean().item() + 1e-5


def _ms(fn, iters=10):
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def test_reference_kernel_speed(ref, cuda_device, no_device_error, capsys):
    """Per-launch time of every reference kernel next to this library's, at the PixAI bs16 shapes of one
    block (M = 16 x 5184 tokens). The reference GEMM takes its faster pipeline depth (its autotuner's
    choice, engine.py:89-119). Prints a table; asserts only that both sides ran."""
    from foidfinder_b200 import ops
    from foidfinder_b200.weights import axial_rope

    d, M = cuda_device, 16 * 5184
    rows = []
    x = _act(M, 1024, 1, d)
    gam, bet = torch.ones(1024, device=d), torch.zeros(1024, device=d)
    q8, rs = torch.empty(M, 1024, dtype=torch.int8, device=d), torch.empty(M, device=d)
    rows.append(("rot_q8_1024 + LN", _ms(lambda: ref.rot_q8_1024(x, gam, bet, q8, rs)),
                 _ms(lambda: ops.rot_q8_1024(x, gam, bet, q8, rs))))
    rows.append(("rot_q8_1024", _ms(lambda: ref.rot_q8_1024(x, None, None, q8, rs)),
                 _ms(lambda: ops.rot_q8_1024(x, None, None, q8, rs))))
    h = _act(M, 4864, 2, d)
    h8 = torch.empty(M, 4864, dtype=torch.int8, device=d)
    hv, h8v = h[:, :4736].contiguous(), torch.empty(M, 4736, dtype=torch.int8, device=d)
    rows.append(("rot_q8_h128 4736 (ours: 4864 padded)", _ms(lambda: ref.rot_q8_h128(hv, h8v, rs)),
                 _ms(lambda: ops.rot_q8_h128(h, h8, rs))))
    del hv, h8v
    cos, sin = (t.contiguous().to(d) for t in axial_rope(24, 1.0))
    cos_t, sin_t = cos.t().contiguous(), sin.t().contiguous()

    def gemm_pair(name, N, K, epi_ref, epi_ours, out_cols, K_ours=None, N_ours=None, rope=False):
        A, W, rsg, csg, bg = _gemm_case(M, N, K, N + K, d)
        out = torch.zeros(M, out_cols, dtype=torch.float16, device=d)
        kw = dict(rope_cos=cos_t, rope_sin=sin_t, rope_cols=2048, tokens=576) if rope else {}
        t_ref = min(_ms(lambda st=st: ref.gemm_s8(A, W, rsg, csg, bg, out, epi_ref, st, cos if rope else None,
                                                  sin if rope else None, Q_SCALE)) for st in (2, 3))
        if K_ours or N_ours:
            A2, W2, rs2, cs2, b2 = _gemm_case(M, N_ours or N, K_ours or K, 1, d)
            out2 = torch.zeros(M, N_ours or out_cols, dtype=torch.float16, device=d)
            t_ours = _ms(lambda: ops.gemm_s8(A2, W2, rs2, cs2, b2, out2, epi_ours, **kw))
        else:
            t_ours = _ms(lambda: ops.gemm_s8(A, W, rsg, csg, bg, out, epi_ours, **kw))
        rows.append((name, t_ref, t_ours))

    gemm_pair("gemm qkv + RoPE (3072 x 1024)", 3072, 1024, 0, ops.EPI_QKV_ROPE, 3072, rope=True)
    gemm_pair("gemm proj + residual (1024 x 1024)", 1024, 1024, 1, ops.EPI_RESIDUAL, 1024)
    gemm_pair("gemm fc1 + GELU (4736 x 1024; ours 4864)", 4736, 1024, 2, ops.EPI_GELU, 4736, N_ours=4864)
    gemm_pair("gemm fc2 + residual (1024 x 4736; ours K 4864)", 1024, 4736, 1, ops.EPI_RESIDUAL, 1024, K_ours=4864)
    for seqs, seq in ((16 * 9, 576), (16, 5184)):
        qkv = (_act(seqs * seq, 3072, 3, d).float() * 0.3).half()
        o = torch.empty(seqs * seq, 1024, dtype=torch.float16, device=d)
        rows.append((f"attention {seqs} x {seq}", _ms(lambda: ref.attention(qkv, o, seq)),
                     _ms(lambda: ops.attention(qkv, o, seq, 16, scale=math.log(2.0)))))
        del qkv, o
    with capsys.disabled():
        print("\nreference kernel vs foidfinder_b200 on B200 (ms per launch, PixAI bs16 block shapes)")
        for name, a, b in rows:
            print(f"  {name:48s} ref {a:8.3f}  ours {b:8.3f}  speed-up {a / b:5.2f}x")
    assert all(a > 0 and b > 0 for _, a, b in rows)
