"""GPU parity tests of the library's kernels through the C ABI (h3k_*), each against the CPU oracle or a plain fp32
restatement of the same operation on the same (bf16-valued) inputs. Integer and index results must match bit for
bit; floating-point results within the tolerance written in each test."""
import ctypes

import numpy as np
import pytest
import torch

import h3b200 as H
from oracle import exact, h3_oracle as O

pytestmark = pytest.mark.gpu


def stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def sync():
    H.check(H.lib().h3k_check(stream()))


def ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def rel(a, b):
    a = a.double().cpu()
    b = b.double().cpu()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def gemm(A, B, args, epi, int8=False):
    H.check(H.lib().h3k_gemm(ptr(A), ptr(B), ctypes.byref(args), epi, 1 if int8 else 0, stream()))
    sync()


def args(**kw):
    a = H.h3k_gemm_args()
    a.a_chunks = 1
    a.eps = 1e-6
    a._keep = [v for v in kw.values() if isinstance(v, torch.Tensor)]  # alive until the GEMM has run
    for k, v in kw.items():
        setattr(a, k, ptr(v) if isinstance(v, torch.Tensor) else v)
    return a


# ------------------------------------------------------------------------------------------------- synthetic

@pytest.mark.parametrize("bf16", [0, 1])
def test_fill_synthetic_bit_exact(cuda, bf16):
    n = 1 << 20
    t = torch.empty(n, dtype=torch.bfloat16 if bf16 else torch.float32, device=cuda)
    H.check(H.lib().h3k_fill_synthetic(ptr(t), bf16, n, 5, 123, 1.0 if bf16 else 0.0, 0.02, stream()))
    sync()
    want = O.synthetic(n, 5, 123, 1.0 if bf16 else 0.0, 0.02, bool(bf16))
    np.testing.assert_array_equal(t.float().cpu().numpy(), want)


# ------------------------------------------------------------------------------------------------------ GEMM

@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (300, 512, 320), (1000, 768, 5120), (77, 256, 96), (4128, 1024, 1024)])
def test_gemm_bf16_f32_out(cuda, M, N, K):
    g = torch.Generator(device="cpu").manual_seed(M + N + K)
    A = torch.randn(M, K, generator=g).bfloat16().to(cuda)
    B = (torch.randn(N, K, generator=g) * 0.05).bfloat16().to(cuda)
    bias = torch.randn(N, generator=g).to(cuda)
    out = torch.zeros(M, N, device=cuda)
    gemm(A, B, args(M=M, N=N, K=K, out=out, ldo=N, bias=bias), H.EPI_F32)
    want = A.float() @ B.float().T + bias
    assert rel(out, want) < 1e-5


def test_gemm_bf16_out_and_lda(cuda):
    M, N, K, lda = 500, 512, 192, 256
    A = torch.randn(M, lda, device=cuda).bfloat16()
    B = torch.randn(N, K, device=cuda).bfloat16()
    out = torch.zeros(M, N, device=cuda, dtype=torch.bfloat16)
    gemm(A, B, args(M=M, N=N, K=K, lda=lda, out=out, ldo=N), H.EPI_BF16)
    want = A[:, :K].float() @ B.float().T
    assert rel(out.float(), want) < 4e-3  # the bf16 rounding of the output


def test_gemm_chunked_a(cuda):
    """A split into P column chunks [chunk][rows][K/P] (the layout after the sequence-parallel all-to-all)."""
    P, M, Kc, N = 4, 300, 256, 512
    chunks = torch.randn(P, M, Kc, device=cuda).bfloat16()
    B = torch.randn(N, P * Kc, device=cuda).bfloat16()
    out = torch.zeros(M, N, device=cuda)
    gemm(chunks, B, args(M=M, N=N, K=P * Kc, a_chunks=P, lda=Kc, a_rows_stride=M, out=out, ldo=N), H.EPI_F32)
    A = chunks.permute(1, 0, 2).reshape(M, P * Kc)
    assert rel(out, A.float() @ B.float().T) < 1e-5


@pytest.mark.parametrize("M,N,K", [(128, 256, 128), (333, 512, 640), (2000, 1024, 5120)])
def test_gemm_int8_bit_exact(cuda, M, N, K):
    """gemm_i8: the int32 dot products are the exact integer sums (the reference's dequant path's integers)."""
    g = torch.Generator(device="cpu").manual_seed(K)
    A = torch.randint(-127, 128, (M, K), generator=g, dtype=torch.int8)
    B = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int8)
    out = torch.zeros(M, N, dtype=torch.int32, device=cuda)
    gemm(A.to(cuda), B.to(cuda), args(M=M, N=N, K=K, out=out, ldo=N), H.EPI_S32, int8=True)
    want = A.numpy().astype(np.int64) @ B.numpy().astype(np.int64).T
    np.testing.assert_array_equal(out.cpu().numpy().astype(np.int64), want)


def test_gemm_int8_dequant(cuda):
    M, N, K = 300, 512, 1024
    x = torch.from_numpy(O.bf16_round(np.random.default_rng(1).standard_normal((M, K)).astype(np.float32)))
    w = torch.from_numpy(O.bf16_round((np.random.default_rng(2).standard_normal((N, K)) * 0.02).astype(np.float32)))
    qa, sa = O.quant_rows(x.numpy())
    qw, sw = O.quant_rows(w.numpy())
    out = torch.zeros(M, N, device=cuda, dtype=torch.bfloat16)
    tq = lambda a: torch.from_numpy(a).to(cuda)
    gemm(tq(qa), tq(qw), args(M=M, N=N, K=K, out=out, ldo=N, a_scale=tq(sa), b_scale=tq(sw)), H.EPI_BF16, int8=True)
    want = O.int8_linear(x, w, torch.zeros(N))
    assert rel(out.float(), want) < 4e-3


def rope_inputs(S, seed=0):
    """A rotary table for S rows at arbitrary (t, h, w) positions."""
    rng = np.random.default_rng(seed + S)
    pos = np.stack([np.arange(S, dtype=np.float64), rng.uniform(-20, 20, S), rng.uniform(-20, 20, S)], 1)
    return torch.from_numpy(O.rope_table(pos))


def test_gemm_qkv_epilogue(cuda):
    """heads_partial fused: q/k per-head RMS norm * weight and the rotary; v plus bias; [rows][3][heads][128]."""
    M, d, Hh = 300, 512, 4
    inner = Hh * 128
    g = torch.Generator().manual_seed(0)
    A = torch.randn(M, d, generator=g).bfloat16()
    B = (torch.randn(3 * inner, d, generator=g) * 0.05).bfloat16()
    bias = torch.randn(3 * inner, generator=g) * 0.1
    qn = 1 + 0.1 * torch.randn(128, generator=g)
    kn = 1 + 0.1 * torch.randn(128, generator=g)
    cs = rope_inputs(M)
    out = torch.zeros(M, 3, Hh, 128, device=cuda, dtype=torch.bfloat16)
    gemm(A.to(cuda), B.to(cuda), args(M=M, N=3 * inner, K=d, out=out, bias=bias.to(cuda), rope=cs.to(cuda), qn_w=qn.to(cuda),
                                      kn_w=kn.to(cuda), inner=inner, heads_per_rank=Hh, rows_local=M), H.EPI_QKV)
    y = (A.float() @ B.float().T + bias).reshape(M, 3, Hh, 128)
    q = O.rope(O.rms(y[:, 0], 1e-6) * qn, cs)
    k = O.rope(O.rms(y[:, 1], 1e-6) * kn, cs)
    assert rel(out[:, 0].float(), q) < 5e-3
    assert rel(out[:, 1].float(), k) < 5e-3
    assert rel(out[:, 2].float(), y[:, 2]) < 5e-3


def test_gemm_qkv_epilogue_head_split_layout(cuda):
    """With P ranks the qkv epilogue writes [P][rows][3][heads/P][128] (the all-to-all's send layout)."""
    M, d, Hh, P = 200, 256, 4, 2
    inner = Hh * 128
    A = torch.randn(M, d, device=cuda).bfloat16()
    B = (torch.randn(3 * inner, d, device=cuda) * 0.05).bfloat16()
    cs = rope_inputs(M).to(cuda)
    ones = torch.ones(128, device=cuda)
    full = torch.zeros(M, 3, Hh, 128, device=cuda, dtype=torch.bfloat16)
    split = torch.zeros(P, M, 3, Hh // P, 128, device=cuda, dtype=torch.bfloat16)
    common = dict(M=M, N=3 * inner, K=d, rope=cs, qn_w=ones, kn_w=ones, inner=inner, rows_local=M)
    gemm(A, B, args(out=full, heads_per_rank=Hh, **common), H.EPI_QKV)
    gemm(A, B, args(out=split, heads_per_rank=Hh // P, **common), H.EPI_QKV)
    for r in range(P):
        assert torch.equal(split[r], full[:, :, r * Hh // P:(r + 1) * Hh // P])


def test_gemm_gate_resid_epilogue(cuda):
    M, N, K = 300, 512, 256
    A = torch.randn(M, K, device=cuda).bfloat16()
    B = (torch.randn(N, K, device=cuda) * 0.05).bfloat16()
    bias = torch.randn(N, device=cuda)
    x0 = torch.randn(M, N, device=cuda)
    mod = torch.randn(5, 6, N, device=cuda)
    midx = torch.randint(0, 5, (M,), device=cuda, dtype=torch.uint8)
    x = x0.clone()
    gemm(A, B, args(M=M, N=N, K=K, x=x, ldx=N, bias=bias, mod=mod, mod_idx=midx, gate_slot=5, dim=N), H.EPI_GATE_RESID)
    want = x0 + mod[midx.long(), 5] * (A.float() @ B.float().T + bias)
    assert rel(x, want) < 1e-5


def test_gemm_swiglu_epilogue(cuda):
    """fc1 stored [gate; value] (architecture.md:112-114) regrouped into 128-row gate/value pairs."""
    M, F, K = 300, 384, 256
    W = (torch.randn(2 * F, K) * 0.05).bfloat16()
    b = torch.randn(2 * F) * 0.1
    perm = []
    for gI in range(F // 128):
        perm += list(range(gI * 128, gI * 128 + 128)) + list(range(F + gI * 128, F + gI * 128 + 128))
    Wi, bi = W[perm].contiguous(), b[perm].contiguous()
    A = torch.randn(M, K).bfloat16()
    out = torch.zeros(M, F, device=cuda, dtype=torch.bfloat16)
    gemm(A.to(cuda), Wi.to(cuda), args(M=M, N=2 * F, K=K, out=out, ldo=F, bias=bi.to(cuda)), H.EPI_SWIGLU)
    gv = A.float() @ W.float().T + b
    want = torch.nn.functional.silu(gv[:, :F]) * gv[:, F:]
    assert rel(out.float(), want) < 5e-3


# ----------------------------------------------------------------------------------------------- row kernels

@pytest.mark.parametrize("M,d", [(333, 1024), (2000, 5120), (1777, 5376)])
def test_rms_mod_rows(cuda, M, d):
    """The modulated RMS norm (a persistent kernel streaming rows through shared memory; the larger cases give every
    warp several rows, so its two row slots are reused) against the fp32 restatement; int8 output bit for bit."""
    x = torch.randn(M, d, device=cuda) * 3
    w = 1 + 0.1 * torch.randn(d, device=cuda)
    mod = torch.randn(6, 6, d, device=cuda) * 0.2
    midx = torch.randint(0, 6, (M,), device=cuda, dtype=torch.uint8)
    want = O.rms(x.cpu(), 1e-6) * w.cpu() * (1 + mod.cpu()[midx.long().cpu(), 4]) + mod.cpu()[midx.long().cpu(), 3]
    outs = {}
    for kind, dt in ((0, torch.bfloat16), (1, torch.float32), (2, torch.int8)):
        o = torch.zeros(M, d, device=cuda, dtype=dt)
        sc = torch.zeros(M, device=cuda)
        H.check(H.lib().h3k_rms_mod(ptr(x), d, M, d, ptr(w), ptr(mod), ptr(midx), 6, 3, 4, 1e-6, kind, ptr(o), d, ptr(sc), stream()))
        sync()
        outs[kind] = (o, sc)
    assert rel(outs[1][0], want) < 1e-5
    assert rel(outs[0][0].float(), want) < 4e-3
    # int8 output = quant_rows_i8 of the bf16 output, bit for bit
    q, s = O.quant_rows(outs[0][0].float().cpu().numpy())
    np.testing.assert_array_equal(outs[2][0].cpu().numpy(), q)
    np.testing.assert_array_equal(outs[2][1].cpu().numpy(), s)


def test_quant_rows_i8_bit_exact(cuda):
    M, K = 257, 3000 - 3000 % 8
    x = (torch.randn(M, K, device=cuda) * torch.rand(M, 1, device=cuda) * 10).bfloat16()
    x[5] = 0
    q = torch.zeros(M, K, dtype=torch.int8, device=cuda)
    s = torch.zeros(M, device=cuda)
    H.check(H.lib().h3k_quant_rows_i8(ptr(x), K, M, K, ptr(q), ptr(s), stream()))
    sync()
    wq, ws = O.quant_rows(x.float().cpu().numpy())
    np.testing.assert_array_equal(q.cpu().numpy(), wq)
    np.testing.assert_array_equal(s.cpu().numpy(), ws)


def test_gate_add_and_swiglu_rows(cuda):
    M, d = 100, 512
    x0 = torch.randn(M, d, device=cuda)
    y = torch.randn(M, d, device=cuda).bfloat16()
    mod = torch.randn(3, 6, d, device=cuda)
    midx = torch.randint(0, 3, (M,), device=cuda, dtype=torch.uint8)
    x = x0.clone()
    H.check(H.lib().h3k_gate_add(ptr(x), d, ptr(y), d, M, d, ptr(mod), ptr(midx), 2, stream()))
    sync()
    assert rel(x, x0 + mod[midx.long(), 2] * y.float()) < 1e-6
    F = 256
    gv = torch.randn(M, 2 * F, device=cuda).bfloat16()
    out = torch.zeros(M, F, device=cuda, dtype=torch.bfloat16)
    H.check(H.lib().h3k_swiglu(ptr(gv), M, F, ptr(out), stream()))
    sync()
    want = torch.nn.functional.silu(gv[:, :F].float()) * gv[:, F:].float()
    assert rel(out.float(), want) < 4e-3


def test_heads_partial_standalone_matches_fused(cuda):
    M, Hh = 200, 3
    qkv = torch.randn(M, 3, Hh, 128, device=cuda).bfloat16()
    qn = 1 + 0.1 * torch.randn(128, device=cuda)
    kn = 1 + 0.1 * torch.randn(128, device=cuda)
    cs = rope_inputs(M).to(cuda)
    t = qkv.clone()
    H.check(H.lib().h3k_heads_partial(ptr(t), M, Hh, ptr(qn), ptr(kn), ptr(cs), 1e-6, stream()))
    sync()
    q = O.rope(O.rms(qkv[:, 0].float().cpu(), 1e-6) * qn.cpu(), cs.cpu())
    assert rel(t[:, 0].float(), q) < 4e-3
    assert torch.equal(t[:, 2], qkv[:, 2])


# ------------------------------------------------------------------------------------------------- attention

def rms_normed_qk(qkv):
    """q and k RMS-normed per head (unit weights), as the step's q/k/v epilogue leaves them; v as it is."""
    x = qkv.float()
    x[:, :2] = x[:, :2] * torch.rsqrt(x[:, :2].pow(2).mean(-1, keepdim=True) + 1e-6)
    return x.bfloat16()


def score_bound(qkv):
    """max |q.k| / sqrt(128) * log2(e) over every row pair and head, from the norms (Cauchy-Schwarz), with room."""
    qn = qkv[:, 0].float().norm(dim=-1).max().item()
    kn = qkv[:, 1].float().norm(dim=-1).max().item()
    return qn * kn / 128 ** 0.5 * 1.4426950408889634 * 1.01 + 0.01


@pytest.mark.parametrize("S,Hh", [(128, 1), (300, 2), (1111, 3), (4096, 2)])
@pytest.mark.parametrize("bounded", [False, True])
def test_attention_dense(cuda, S, Hh, bounded):
    """Against fp32 softmax; bounded: q and k RMS-normed per head (as the step makes them) and their score bound
    given, so the softmax takes the bound for the row maximum."""
    g = torch.Generator().manual_seed(S)
    qkv = torch.randn(S, 3, Hh, 128, generator=g).bfloat16()
    qkv[:, :2] *= 1.5
    if bounded:
        qkv = rms_normed_qk(qkv)
    t = qkv.to(cuda)
    out = torch.zeros(S, Hh, 128, device=cuda, dtype=torch.bfloat16)
    if bounded:
        bound = score_bound(qkv)
        assert bound < 20
        H.check(H.lib().h3k_attention_bounded(ptr(t[:, 0]), ptr(t[:, 1]), ptr(t[:, 2]), 3 * Hh * 128, Hh, S, bound, ptr(out), Hh * 128,
                                              stream()))
    else:
        H.check(H.lib().h3k_attention(ptr(t[:, 0]), ptr(t[:, 1]), ptr(t[:, 2]), 3 * Hh * 128, Hh, S, ptr(out), Hh * 128, stream()))
    sync()
    want = O.attention(qkv[:, 0].float(), qkv[:, 1].float(), qkv[:, 2].float())
    r = rel(out.float(), want)
    _, cos = O.diff(out.float().cpu().numpy(), want.numpy(), 128)
    assert r < 1e-2 and cos > 0.999, (r, cos)


def sparse_case(cuda, dense_rows=70, frames=5, ph=6, pw=7, Hh=2, seed=0):
    S = dense_rows + frames * ph * pw
    g = torch.Generator().manual_seed(seed)
    base = torch.randn(frames * ph * pw, Hh, 128, generator=g)
    # smooth video rows so cube means differ
    qkv = torch.randn(S, 3, Hh, 128, generator=g)
    qkv[dense_rows:, 0] += 2 * base
    qkv[dense_rows:, 1] += 2 * base.roll(7, 0)
    return qkv.bfloat16(), H.h3k_cube_grid(dense_rows, frames, ph, pw)


def packed(grid):
    """(order, inverse): the sparse calls take rows in the packed order, packed row i = layout row order[i]."""
    order = torch.from_numpy(H.packed_order(grid.dense_rows, grid.frames, grid.ph, grid.pw))
    return order, torch.argsort(order)


@pytest.mark.parametrize("ratio,local", [(0.1, 1), (0.3, 3), (0.5, 0), (1.0, 0)])
def test_sparse_selection_bit_exact(cuda, ratio, local):
    """cube_pool, cube_scores and cube_topk against the exact CPU restatement: identical means, scores, indices."""
    qkv, grid = sparse_case(cuda)
    Hh = qkv.shape[2]
    order, _ = packed(grid)
    t = qkv[order].contiguous().to(cuda)
    nc, kcap = ctypes.c_int32(), ctypes.c_int32()
    H.check(H.lib().h3k_sparse_sizes(ctypes.byref(grid), ratio, local, ctypes.byref(nc), ctypes.byref(kcap), None, None))
    nc, kcap = nc.value, kcap.value
    mq = torch.zeros(Hh, nc, 128, device=cuda)
    mk = torch.zeros(Hh, nc, 128, device=cuda)
    sc = torch.zeros(Hh, nc, nc, device=cuda)
    sel = torch.full((Hh, nc, kcap), -1, dtype=torch.int32, device=cuda)
    nsel = torch.zeros(Hh, nc, dtype=torch.int32, device=cuda)
    H.check(H.lib().h3k_sparse_select(ptr(t[:, 0]), ptr(t[:, 1]), 3 * Hh * 128, Hh, ctypes.byref(grid), ratio, local, ptr(mq), ptr(mk),
                                      ptr(sc), ptr(sel), ptr(nsel), stream()))
    sync()
    bits = lambda a: a.contiguous().view(torch.int16).numpy().view(np.uint16).reshape(-1)
    q_bits = bits(qkv)  # the whole [S][3][H][128] tensor; q at offset 0, k at H*128, row stride 3*H*128
    emq, emk = exact.cube_pool(q_bits, q_bits[Hh * 128:], 3 * Hh * 128, Hh, grid.dense_rows, grid.frames, grid.ph, grid.pw)
    np.testing.assert_array_equal(mq.cpu().numpy(), emq)
    np.testing.assert_array_equal(mk.cpu().numpy(), emk)
    es = exact.cube_scores(emq, emk)
    np.testing.assert_array_equal(sc.cpu().numpy(), es)
    esel, ensel = exact.cube_topk(es, grid.frames, grid.ph, grid.pw, ratio, local)
    np.testing.assert_array_equal(nsel.cpu().numpy(), ensel)
    got = sel.cpu().numpy()
    for h in range(Hh):
        for i in range(nc):
            assert list(got[h, i, :ensel[h, i]]) == list(esel[h, i, :ensel[h, i]]), (h, i)


def allowed_mask(S, D, frames, ph, pw, sel, nsel):
    """[H][S][S]: dense-row queries see every key; a video query in cube c sees its selected cubes' rows and the
    dense rows (architecture.md:126-128)."""
    Hh, nc, _ = sel.shape
    ncy, ncx = (ph + 3) // 4, (pw + 3) // 4
    cube_of = np.zeros(S, np.int64)
    for r in range(D, S):
        v = r - D
        f, y, x = v // (ph * pw), (v // pw) % ph, v % pw
        cube_of[r] = ((f // 4) * ncy + y // 4) * ncx + x // 4
    allowed = np.zeros((Hh, S, S), bool)
    allowed[:, :D, :] = True
    allowed[:, D:, :D] = True
    for h in range(Hh):
        ok = np.zeros((nc, nc), bool)
        for c in range(nc):
            ok[c, sel[h, c, :nsel[h, c]]] = True
        allowed[h, D:, D:] = ok[cube_of[D:]][:, cube_of[D:]]
    return torch.from_numpy(allowed)


@pytest.mark.parametrize("ratio,local", [(0.1, 1), (0.4, 3), (1.0, 0)])
def test_sparse_attention(cuda, ratio, local):
    qkv, grid = sparse_case(cuda, seed=1)
    S, _, Hh, _ = qkv.shape
    order, inverse = packed(grid)
    t = qkv[order].contiguous().to(cuda)
    out_packed = torch.zeros(S, Hh, 128, device=cuda, dtype=torch.bfloat16)
    H.check(H.lib().h3k_sparse_attention(ptr(t[:, 0]), ptr(t[:, 1]), ptr(t[:, 2]), 3 * Hh * 128, Hh, ctypes.byref(grid), ratio, local,
                                         ptr(out_packed), Hh * 128, stream()))
    sync()
    out = out_packed.cpu()[inverse]
    bits = qkv.contiguous().view(torch.int16).numpy().view(np.uint16).reshape(-1)
    mq, mk = exact.cube_pool(bits, bits[Hh * 128:], 3 * Hh * 128, Hh, grid.dense_rows, grid.frames, grid.ph, grid.pw)
    sel, nsel = exact.cube_topk(exact.cube_scores(mq, mk), grid.frames, grid.ph, grid.pw, ratio, local)
    allowed = allowed_mask(S, grid.dense_rows, grid.frames, grid.ph, grid.pw, sel, nsel)
    want = O.attention(qkv[:, 0].float(), qkv[:, 1].float(), qkv[:, 2].float(), allowed)
    r = rel(out.float(), want)
    assert r < 1e-2, r
    if ratio == 1.0:
        dense = torch.zeros_like(out_packed)
        H.check(H.lib().h3k_attention(ptr(t[:, 0]), ptr(t[:, 1]), ptr(t[:, 2]), 3 * Hh * 128, Hh, S, ptr(dense), Hh * 128, stream()))
        sync()
        assert rel(out_packed.float(), dense.float()) < 1e-2  # every cube selected = dense (tests/CMakeLists.txt:9-12)


@pytest.mark.parametrize("ratio,local", [(0.1, 1), (0.4, 3), (1.0, 0)])
def test_sparse_attention_bounded(cuda, ratio, local):
    """The sparse kernel given the score bound (no running maximum, no per-step exchange between a row's warps)
    against the masked fp32 oracle and against the online-maximum kernel on the same selection; ratio 1 against
    dense attention."""
    qkv, grid = sparse_case(cuda, seed=2)
    qkv = rms_normed_qk(qkv)
    S, _, Hh, _ = qkv.shape
    bound = score_bound(qkv)
    assert 10 < bound < 20
    order, inverse = packed(grid)
    t = qkv[order].contiguous().to(cuda)
    L = H.lib()
    outs = []
    for fn, extra in ((L.h3k_sparse_attention_bounded, [bound]), (L.h3k_sparse_attention, [])):
        o = torch.zeros(S, Hh, 128, device=cuda, dtype=torch.bfloat16)
        H.check(fn(ptr(t[:, 0]), ptr(t[:, 1]), ptr(t[:, 2]), 3 * Hh * 128, Hh, ctypes.byref(grid), ratio, local, *extra, ptr(o), Hh * 128,
                   stream()))
        outs.append(o)
    sync()
    out = outs[0].cpu()[inverse]
    bits = qkv.contiguous().view(torch.int16).numpy().view(np.uint16).reshape(-1)
    mq, mk = exact.cube_pool(bits, bits[Hh * 128:], 3 * Hh * 128, Hh, grid.dense_rows, grid.frames, grid.ph, grid.pw)
    sel, nsel = exact.cube_topk(exact.cube_scores(mq, mk), grid.frames, grid.ph, grid.pw, ratio, local)
    allowed = allowed_mask(S, grid.dense_rows, grid.frames, grid.ph, grid.pw, sel, nsel)
    want = O.attention(qkv[:, 0].float(), qkv[:, 1].float(), qkv[:, 2].float(), allowed)
    assert rel(out.float(), want) < 1e-2
    a, b = out.double().reshape(-1, 128), want.double().reshape(-1, 128)
    assert float(((a * b).sum(-1) / (a.norm(dim=-1) * b.norm(dim=-1)).clamp_min(1e-30)).min()) > 0.999
    assert rel(outs[0].float(), outs[1].float()) < 1e-2
    if ratio == 1.0:
        dense = torch.zeros_like(outs[0])
        H.check(L.h3k_attention(ptr(t[:, 0]), ptr(t[:, 1]), ptr(t[:, 2]), 3 * Hh * 128, Hh, S, ptr(dense), Hh * 128, stream()))
        sync()
        assert rel(outs[0].float(), dense.float()) < 1e-2


def test_sparse_attention_bounded_refuses_a_bound_past_its_limit(cuda):
    qkv, grid = sparse_case(cuda)
    S, _, Hh, _ = qkv.shape
    t = qkv.to(cuda)
    o = torch.zeros(S, Hh, 128, device=cuda, dtype=torch.bfloat16)
    for bad in (41.0, -1.0, float("nan")):
        rc = H.lib().h3k_sparse_attention_bounded(ptr(t[:, 0]), ptr(t[:, 1]), ptr(t[:, 2]), 3 * Hh * 128, Hh, ctypes.byref(grid), 0.1, 1,
                                                  bad, ptr(o), Hh * 128, stream())
        assert rc == H.H3_ERR_ARG
        assert "bound" in H.lib().h3_last_error().decode()


# ---------------------------------------------------------------------------------- time embedding and AdaLN

def test_time_mlp_adaln_and_heads(cuda):
    cfg = dict(dim=256, heads=2, ffn=256, blocks=2, time_dim=128, text_dim=256)
    w = O.make_weights(cfg, 3)
    levels = [0.7, 0.3, 0.999]
    temb, s = O.time_embedding(levels, w)
    emb = np.zeros((3, 256), np.float32)
    for u, t in enumerate(levels):
        for i in range(128):
            fr = np.float32(np.exp(-np.log(10000.0) * i / 128.0))
            a = np.float32(t) * fr
            emb[u, i], emb[u, 128 + i] = np.float32(np.cos(float(a))), np.float32(np.sin(float(a)))
    keep = []  # device copies stay referenced until the kernels have run

    def c(t):
        keep.append(t.contiguous().to(cuda))
        return keep[-1]

    h = torch.zeros(3, 256, device=cuda)
    te = torch.zeros(3, 128, device=cuda)
    ts = torch.zeros(3, 128, device=cuda)
    H.check(H.lib().h3k_gemv_f32(ptr(c(w["t_in_w"])), ptr(c(w["t_in_b"])), ptr(c(torch.from_numpy(emb))), 3, 256, 256, 1, ptr(h), None,
                                 stream()))
    H.check(H.lib().h3k_gemv_f32(ptr(c(w["t_out_w"])), ptr(c(w["t_out_b"])), ptr(h), 3, 128, 256, 0, ptr(te), ptr(ts), stream()))
    sync()
    assert rel(te, temb) < 1e-5
    assert (ts.cpu() != s).float().mean() < 0.02  # bf16 rounding of values within an ulp may differ
    W = torch.cat([b["ada_w"] for b in w["blocks"]]).bfloat16()
    bb = torch.cat([b["ada_b"] for b in w["blocks"]])
    mods = torch.zeros(2 * 3 * 18 * 256, device=cuda)
    H.check(H.lib().h3k_adaln(ptr(c(W)), ptr(c(bb)), ptr(c(s)), 3, 2, 18 * 256, 128, ptr(mods), stream()))
    sync()
    want = torch.stack([s @ b["ada_w"].T + b["ada_b"] for b in w["blocks"]])  # [L][U][18 d]
    assert rel(mods.view(2, 3, -1), want) < 1e-5
    x = torch.randn(200, 256)
    out = torch.zeros(200, 128, device=cuda)
    H.check(H.lib().h3k_heads(ptr(c(x)), 256, 200, ptr(c(w["hv_w"])), ptr(c(w["hv_b"])), 96, 256, ptr(out), 128, stream()))
    sync()
    assert rel(out[:, :96], x @ w["hv_w"].T + w["hv_b"]) < 1e-5


def test_host_pointers_are_refused_before_any_launch(cuda):
    """A plain host buffer handed to a kernel entry point is an argument error, not a kernel fault."""
    Hh, S = 2, 128
    t = torch.zeros(S, 3, Hh, 128, device=cuda, dtype=torch.bfloat16)
    host_out = np.zeros((S, Hh, 128), np.uint16)
    rc = H.lib().h3k_attention(ptr(t[:, 0]), ptr(t[:, 1]), ptr(t[:, 2]), 3 * Hh * 128, Hh, S, ctypes.c_void_p(host_out.ctypes.data),
                               Hh * 128, stream())
    assert rc == H.H3_ERR_ARG
    assert b"host memory" in H.lib().h3_last_error()
    grid = H.h3k_cube_grid(64, 4, 4, 4)
    rc = H.lib().h3k_sparse_attention(ctypes.c_void_p(host_out.ctypes.data), ptr(t[:, 1]), ptr(t[:, 2]), 3 * Hh * 128, Hh,
                                      ctypes.byref(grid), 0.5, 1, ptr(t[:, 0]), Hh * 128, stream())
    assert rc == H.H3_ERR_ARG
    sync()  # the context is intact


def test_bounded_wait_gives_up_and_the_context_survives(cuda):
    """Failure detection without a GPU fault: a wait on an mbarrier nothing arrives on runs out after its cycle budget
    (~1 ms here), the kernel ends, the host reads H3_ERR_DEVICE, and the next kernels run normally."""
    import time
    t0 = time.time()
    rc = H.lib().h3k_wait_selftest(2_000_000, stream())
    assert rc == H.H3_ERR_DEVICE, rc
    assert b"ran out" in H.lib().h3_last_error()
    assert time.time() - t0 < 10
    sync()  # the error word was cleared: h3k_check reports nothing
    S, Hh = 256, 2
    t = (torch.randn(S, 3, Hh, 128, device=cuda)).bfloat16()
    out = torch.zeros(S, Hh, 128, device=cuda, dtype=torch.bfloat16)
    H.check(H.lib().h3k_attention(ptr(t[:, 0]), ptr(t[:, 1]), ptr(t[:, 2]), 3 * Hh * 128, Hh, S, ptr(out), Hh * 128, stream()))
    sync()
    want = O.attention(t[:, 0].float().cpu(), t[:, 1].float().cpu(), t[:, 2].float().cpu(), None)
    assert rel(out.float().cpu(), want) < 1e-2
