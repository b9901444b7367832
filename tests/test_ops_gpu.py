"""Numerics of every sm_100a kernel against an fp32 PyTorch reference of the same op."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu

from accerl_agent_b200 import ops
from accerl_agent_b200.algo.objectives import ObjectiveConfig, varlen_token_sum_loss
from accerl_agent_b200.ops import reference as ref

DEV = "cuda"


def _rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


@pytest.fixture(autouse=True)
def _seed():
    torch.manual_seed(0)
    yield
    ops.check_status(torch.device(DEV))


@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, False), (True, True)])
@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (300, 264, 136), (1024, 768, 1536)])
def test_gemm_layouts(a_mn, b_mn, M, N, K):
    if a_mn and M % 8:
        # an MN-major A is stored [K, M]; TMA needs its row stride to be a multiple of 16 bytes
        a_in = torch.zeros(K, M, device=DEV).bfloat16()
        with pytest.raises(RuntimeError):
            ops.gemm(a_in, torch.zeros(N, K, device=DEV).bfloat16(), a_mn=True)
        return
    A = torch.randn(M, K, device=DEV).bfloat16()
    B = torch.randn(N, K, device=DEV).bfloat16()
    a_in = A.t().contiguous() if a_mn else A
    b_in = B.t().contiguous() if b_mn else B
    out = ops.gemm(a_in, b_in, a_mn=a_mn, b_mn=b_mn, out_dtype=torch.float32)
    want = A.float() @ B.float().t()
    assert _rel(out, want) < 1e-5
    out_bf = ops.gemm(a_in, b_in, a_mn=a_mn, b_mn=b_mn)
    assert _rel(out_bf, want) < 1e-2


@pytest.mark.parametrize("block_n", [128, 256])
def test_gemm_epilogue_bias_residual_beta(block_n):
    M, N, K = 520, 1024, 320
    A = torch.randn(M, K, device=DEV).bfloat16()
    B = torch.randn(N, K, device=DEV).bfloat16()
    bias = torch.randn(N, device=DEV).bfloat16()
    res = torch.randn(M, N, device=DEV).bfloat16()
    out = ops.gemm(A, B, bias=bias, residual=res, block_n=block_n)
    want = A.float() @ B.float().t() + bias.float() + res.float()
    assert _rel(out, want) < 1e-2
    acc = torch.randn(M, N, device=DEV)
    base = acc.clone()
    ops.gemm(A, B, acc, beta=1.0, alpha=0.5, out_dtype=torch.float32, block_n=block_n)
    assert _rel(acc, base + 0.5 * (A.float() @ B.float().t())) < 1e-5


@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, True), (True, False)])
@pytest.mark.parametrize("M,N,K", [(1024, 1536, 512), (520, 776, 328)])
def test_gemm_cta_pair_layouts(a_mn, b_mn, M, N, K):
    """The CTA-pair kernel (two SMs per 256 x 256 tile, tcgen05 cta_group::2) for every operand
    major, with row / column / K tails, against the fp32 product."""
    A = torch.randn(M, K, device=DEV).bfloat16()
    B = torch.randn(N, K, device=DEV).bfloat16()
    a_in = A.t().contiguous() if a_mn else A
    b_in = B.t().contiguous() if b_mn else B
    want = A.float() @ B.float().t()
    out = ops.gemm(a_in, b_in, a_mn=a_mn, b_mn=b_mn, out_dtype=torch.float32, block_n=-256)
    assert _rel(out, want) < 1e-5
    out_bf = ops.gemm(a_in, b_in, a_mn=a_mn, b_mn=b_mn, block_n=-256)
    assert _rel(out_bf, want) < 1e-2
    st = ops.status_tensor(torch.device(DEV))
    assert int(st[0]) == 0


def test_gemm_cta_pair_epilogues_and_split():
    M, N, K = 777, 1280, 1024
    A = torch.randn(M, K, device=DEV).bfloat16()
    B = torch.randn(N, K, device=DEV).bfloat16()
    bias = torch.randn(N, device=DEV).bfloat16()
    res = torch.randn(M, N, device=DEV).bfloat16()
    out = ops.gemm(A, B, bias=bias, residual=res, block_n=-256)
    assert _rel(out, A.float() @ B.float().t() + bias.float() + res.float()) < 1e-2
    acc = torch.randn(M, N, device=DEV)
    base = acc.clone()
    ops.gemm(A, B, acc, beta=1.0, alpha=0.5, out_dtype=torch.float32, block_n=-256)
    assert _rel(acc, base + 0.5 * (A.float() @ B.float().t())) < 1e-5
    acc2 = torch.zeros(M, N, device=DEV)
    ops.gemm(A, B, acc2, beta=1.0, out_dtype=torch.float32, block_n=-256, splits=4)
    assert _rel(acc2, A.float() @ B.float().t()) < 1e-5
    # a grid smaller than the tile count: clusters loop over several work items
    out3 = ops.gemm(A, B, block_n=-256, max_ctas=4)
    assert _rel(out3, A.float() @ B.float().t()) < 1e-2


@pytest.mark.parametrize("block_n", [256, -256])
@pytest.mark.parametrize("M,I,K", [(520, 384, 320), (1024, 256, 192)])
def test_gemm_swiglu_epilogues(block_n, M, I, K):
    """Gate/up GEMM with the SwiGLU epilogue (single CTA and CTA pair) and the down-projection dgrad
    with the SwiGLU-backward epilogue, against the fp32 reference and the unfused kernels."""
    x = torch.randn(M, K, device=DEV).bfloat16()
    w = (torch.randn(2 * I, K, device=DEV) * 0.1).bfloat16()
    h = torch.empty(M, I, device=DEV, dtype=torch.bfloat16)
    gu = torch.empty(M, 2 * I, device=DEV, dtype=torch.bfloat16)
    st = ops.status_tensor(torch.device(DEV))
    ops.native().gemm_glu(x, w, gu, h, st, block_n, 0)
    want_gu = x.float() @ w.float().t()
    assert _rel(gu, want_gu) < 1e-2
    assert torch.equal(h, ops.swiglu(gu))  # the epilogue's SwiGLU is the kernel's, bit for bit
    h2 = torch.empty_like(h)
    ops.native().gemm_glu(x, w, None, h2, st, block_n, 0)
    assert torch.equal(h2, h)
    wd = (torch.randn(K, I, device=DEV) * 0.1).bfloat16()  # down projection [out=K, I]
    dy = torch.randn(M, K, device=DEV).bfloat16()
    dgu = torch.empty_like(gu)
    ops.native().gemm_dglu(dy, wd, gu, dgu, st, block_n, 0)
    da = ops.gemm(dy, wd, b_mn=True, block_n=block_n)
    ref = ops.swiglu_backward(da, gu)
    assert _rel(dgu, ref) < 1e-2
    g, u = gu.float()[:, :I], gu.float()[:, I:]
    sig = torch.sigmoid(g)
    d = (dy.float() @ wd.float())
    want = torch.cat([d * u * sig * (1 + g * (1 - sig)), d * (g * sig)], 1)
    assert _rel(dgu, want) < 2e-2
    assert int(st[0]) == 0
    # the public wrappers
    hh, gg = ops.linear_swiglu(x, w, keep_gu=True)
    assert _rel(gg, want_gu) < 1e-2 and _rel(hh, ops.swiglu(gg)) < 1e-6
    assert _rel(ops.linear_dgrad_swiglu(dy, wd, gu), ref) < 1e-2


def test_gemm_strided_views():
    # q/k/v style column slices of a fused buffer as operands and outputs
    T, H = 384, 256
    qkv = torch.randn(T, 3 * H, device=DEV).bfloat16()
    W = torch.randn(H, H, device=DEV).bfloat16()
    q = qkv[:, H : 2 * H]
    out = torch.empty(T, 2 * H, device=DEV, dtype=torch.bfloat16)
    ops.gemm(q, W, out[:, H:])
    assert _rel(out[:, H:], q.float() @ W.float().t()) < 1e-2


def test_linear_grads_match_autograd():
    T, IN, OUT = 640, 512, 384
    x = torch.randn(T, IN, device=DEV).bfloat16()
    w = (torch.randn(OUT, IN, device=DEV) * 0.05).bfloat16()
    dy = torch.randn(T, OUT, device=DEV).bfloat16()
    xf = x.float().requires_grad_(True)
    wf = w.float().requires_grad_(True)
    (xf @ wf.t()).backward(dy.float())
    dx = ops.linear_dgrad(dy, w)
    gw = torch.zeros(OUT, IN, device=DEV)
    ops.linear_wgrad(dy, x, gw, accumulate=True)
    ops.linear_wgrad(dy, x, gw, accumulate=True)
    assert _rel(dx, xf.grad) < 1e-2
    assert _rel(gw, 2 * wf.grad) < 1e-5
    db = torch.zeros(OUT, device=DEV)
    ops.bias_grad(dy, db)
    assert _rel(db, dy.float().sum(0)) < 1e-5


def test_rmsnorm_fwd_bwd():
    T, H = 777, 1536
    x = torch.randn(T, H, device=DEV).bfloat16()
    w = (1 + 0.1 * torch.randn(H, device=DEV)).bfloat16()
    y, rstd = ops.rmsnorm(x, w, 1e-6)
    y_ref, rstd_ref = ref.rmsnorm(x, w, 1e-6)
    assert _rel(y, y_ref) < 1e-2
    assert _rel(rstd, rstd_ref) < 1e-5
    dy = torch.randn(T, H, device=DEV).bfloat16()
    acc = torch.randn(T, H, device=DEV).bfloat16()
    dw = torch.zeros(H, device=DEV)
    dx = ops.rmsnorm_backward(dy, x, w, rstd, dx_accum=acc, dw_grad=dw)
    dx_ref, dw_ref = ref.rmsnorm_backward(dy, x, w, rstd_ref)
    assert _rel(dx, dx_ref + acc.float()) < 1e-2
    assert _rel(dw, dw_ref) < 1e-2


def test_rope_roundtrip_and_reference():
    T, Hq, Hkv, D = 300, 12, 2, 128
    qkv = torch.randn(T, (Hq + 2 * Hkv) * D, device=DEV).bfloat16()
    pos = torch.randint(0, 8192, (T,), device=DEV)
    orig = qkv.clone()
    ops.rope_(qkv, pos, Hq + Hkv, D, 1e6)
    want = ref.apply_rope(orig[:, : (Hq + Hkv) * D].reshape(T, Hq + Hkv, D), pos, 1e6)
    assert _rel(qkv[:, : (Hq + Hkv) * D].reshape(T, Hq + Hkv, D), want) < 1e-2
    assert torch.equal(qkv[:, (Hq + Hkv) * D :], orig[:, (Hq + Hkv) * D :])
    ops.rope_(qkv, pos, Hq + Hkv, D, 1e6, inverse=True)
    assert _rel(qkv, orig) < 2e-2


def test_swiglu_fwd_bwd():
    T, I = 513, 8960
    gu = torch.randn(T, 2 * I, device=DEV).bfloat16()
    h = ops.swiglu(gu)
    assert _rel(h, ref.swiglu(gu)) < 1e-2
    dh = torch.randn(T, I, device=DEV).bfloat16()
    assert _rel(ops.swiglu_backward(dh, gu), ref.swiglu_backward(dh, gu)) < 1e-2


def test_embedding_fwd_bwd():
    V, H, T = 5000, 1536, 1000
    table = torch.randn(V, H, device=DEV).bfloat16()
    ids = torch.randint(0, V, (T,), device=DEV)
    out = ops.embedding(ids, table)
    assert torch.equal(out, table[ids])
    d = torch.randn(T, H, device=DEV).bfloat16()
    g = torch.zeros(V, H, device=DEV)
    ops.embedding_backward(ids, d, g)
    want = torch.zeros(V, H, device=DEV).index_add_(0, ids, d.float())
    assert _rel(g, want) < 1e-5


def test_logsoftmax_label_fwd_bwd():
    n, V = 37, 151936
    logits = (torch.randn(n, V, device=DEV) * 3).bfloat16()
    labels = torch.randint(0, V, (n,), device=DEV)
    lp, lse, ent = ops.logsoftmax_label(logits, labels, with_entropy=True)
    lp_r, lse_r, ent_r = ref.logsoftmax_label(logits, labels)
    assert torch.allclose(lp, lp_r, atol=2e-3, rtol=0)
    assert torch.allclose(lse, lse_r, atol=2e-3, rtol=0)
    assert torch.allclose(ent, ent_r, atol=2e-2, rtol=1e-3)
    g = torch.randn(n, device=DEV)
    lf = logits.float().requires_grad_(True)
    (torch.log_softmax(lf, -1).gather(1, labels.view(-1, 1)).squeeze(1) * g).sum().backward()
    d = logits.clone()
    ops.logsoftmax_label_backward(d, labels, lse, g)
    assert _rel(d, lf.grad) < 1e-2


@pytest.mark.parametrize("mode", ["ppo", "gipo", "sapo", "none"])
def test_policy_loss_matches_autograd(mode):
    n = 5000
    lp = -torch.rand(n, device=DEV) * 5
    old = lp + 0.3 * torch.randn(n, device=DEV)
    adv = torch.randn(n, device=DEV)
    cfg = ObjectiveConfig(clip_mode=mode, clip_eps=0.2, kl_coef=0.05)
    dlp, stats = ops.policy_loss(lp, old, adv, cfg, loss_scale=0.25)
    x = lp.clone().requires_grad_(True)
    loss, stats_ref = varlen_token_sum_loss(x, old, adv, cfg)
    (loss * 0.25).backward()
    assert torch.allclose(dlp, x.grad, atol=1e-5, rtol=1e-4)
    assert torch.allclose(stats, stats_ref.to(stats.device), rtol=1e-4, atol=1e-2)


def test_adamw_matches_torch():
    n = 10007
    p0 = torch.randn(n, device=DEV)
    grads = [torch.randn(n, device=DEV) * 3 for _ in range(3)]
    ref_p = p0.clone().requires_grad_(True)
    opt = torch.optim.AdamW([ref_p], lr=1e-3, weight_decay=0.01)
    master, m, v = p0.clone(), torch.zeros(n, device=DEV), torch.zeros(n, device=DEV)
    bf = torch.empty(n, device=DEV, dtype=torch.bfloat16)
    for step, g in enumerate(grads, start=1):
        ref_p.grad = g.clone()
        torch.nn.utils.clip_grad_norm_([ref_p], 1.0)
        opt.step()
        gg = g.clone()
        ss = ops.grad_sumsq(gg)
        ops.adamw_step(master, m, v, gg, bf, ss, 1e-3, 0.9, 0.999, 1e-8, 0.01, 1.0, step)
        assert float(gg.abs().max()) == 0.0
    assert torch.allclose(master, ref_p.detach(), atol=1e-6, rtol=1e-5)
    assert torch.equal(bf, master.bfloat16())


def _varlen_case(lengths, Hq, Hkv, D=128):
    T = sum(lengths)
    cu = torch.tensor([0] + list(torch.tensor(lengths).cumsum(0)), dtype=torch.int32, device=DEV)
    qkv = (torch.randn(T, (Hq + 2 * Hkv) * D, device=DEV)).bfloat16()
    q = qkv[:, : Hq * D]
    k = qkv[:, Hq * D : (Hq + Hkv) * D]
    v = qkv[:, (Hq + Hkv) * D :]
    return T, cu, qkv, q, k, v


@pytest.mark.parametrize("lengths,Hq,Hkv", [([1, 130, 257, 64], 4, 2), ([512], 2, 2), ([300, 700], 6, 1)])
def test_attention_forward(lengths, Hq, Hkv):
    T, cu, qkv, q, k, v = _varlen_case(lengths, Hq, Hkv)
    o, lse = ops.attention_varlen(q, k, v, cu, max(lengths), Hq, Hkv, 128)
    o_r, lse_r = ref.attention_varlen(q.reshape(T, Hq, 128), k.reshape(T, Hkv, 128), v.reshape(T, Hkv, 128), cu,
                                      1 / math.sqrt(128))
    assert _rel(o, o_r.reshape(T, -1)) < 2e-2
    assert torch.allclose(lse, lse_r, atol=1e-2)


@pytest.mark.parametrize("lengths,Hq,Hkv", [([1, 130, 257, 64], 4, 2), ([384], 2, 2), ([300, 700], 6, 1)])
def test_attention_backward(lengths, Hq, Hkv):
    T, cu, qkv, q, k, v = _varlen_case(lengths, Hq, Hkv)
    o, lse = ops.attention_varlen(q, k, v, cu, max(lengths), Hq, Hkv, 128)
    do = torch.randn(T, Hq * 128, device=DEV).bfloat16()
    dq, dk, dv = ops.attention_varlen_backward(do, q, k, v, o, lse, cu, max(lengths), Hq, Hkv, 128)
    qf = q.float().reshape(T, Hq, 128).requires_grad_(True)
    kf = k.float().reshape(T, Hkv, 128).requires_grad_(True)
    vf = v.float().reshape(T, Hkv, 128).requires_grad_(True)
    of, _ = ref.attention_varlen(qf, kf, vf, cu, 1 / math.sqrt(128))
    of.backward(do.float().reshape(T, Hq, 128))
    assert _rel(dq, qf.grad.reshape(T, -1)) < 3e-2
    assert _rel(dk, kf.grad.reshape(T, -1)) < 3e-2
    assert _rel(dv, vf.grad.reshape(T, -1)) < 3e-2


def test_attention_forward_paged_keys():
    """Prefill queries over keys read in place from a paged cache (one TMA box per page) equal the
    same attention over the keys gathered into contiguous rows."""
    Hq, Hkv, D, bs = 6, 2, 128, 16
    q_lens, k_lens = [37, 130, 1], [300, 130, 515]
    nb = 96
    kc = torch.randn(nb, bs, Hkv, D, device=DEV).bfloat16()
    vc = torch.randn(nb, bs, Hkv, D, device=DEV).bfloat16()
    perm = torch.randperm(nb, device=DEV).to(torch.int32)
    max_blocks = max((n + bs - 1) // bs for n in k_lens)
    table = torch.zeros(len(k_lens), max_blocks, dtype=torch.int32, device=DEV)
    used = 0
    rows = []
    for b, n in enumerate(k_lens):
        nblk = (n + bs - 1) // bs
        table[b, :nblk] = perm[used : used + nblk]
        used += nblk
        pk = torch.arange(n, device=DEV)
        rows.append(table[b, pk // bs].long() * bs + pk % bs)
    idx = torch.cat(rows)
    kctx = kc.view(-1, Hkv * D).index_select(0, idx)
    vctx = vc.view(-1, Hkv * D).index_select(0, idx)
    cu_q = torch.tensor([0] + list(torch.tensor(q_lens).cumsum(0)), dtype=torch.int32, device=DEV)
    cu_k = torch.tensor([0] + list(torch.tensor(k_lens).cumsum(0)), dtype=torch.int32, device=DEV)
    q = torch.randn(sum(q_lens), Hq * D, device=DEV).bfloat16()
    want, lse_w = ops.attention_varlen(q, kctx, vctx, cu_q, max(q_lens), Hq, Hkv, D, cu_seqlens_k=cu_k)
    got, lse_g = ops.attention_varlen(q, kc, vc, cu_q, max(q_lens), Hq, Hkv, D, cu_seqlens_k=cu_k, block_table=table)
    assert torch.equal(got, want)
    assert torch.allclose(lse_g, lse_w)


def test_attention_backward_fused_inverse_rope():
    """The finishing kernel's fused inverse rotation equals the separate RoPE kernel run afterwards."""
    lengths, Hq, Hkv = [200, 333], 6, 2
    T, cu, qkv, q, k, v = _varlen_case(lengths, Hq, Hkv)
    o, lse = ops.attention_varlen(q, k, v, cu, max(lengths), Hq, Hkv, 128)
    do = torch.randn(T, Hq * 128, device=DEV).bfloat16()
    pos = torch.cat([torch.arange(n, device=DEV) for n in lengths]).long()
    dq, dk, dv = ops.attention_varlen_backward(do, q, k, v, o, lse, cu, max(lengths), Hq, Hkv, 128)
    d = torch.cat([dq, dk, dv], 1)
    ops.rope_(d, pos, Hq + Hkv, 128, 1e6, inverse=True)
    fq, fk, fv = ops.attention_varlen_backward(do, q, k, v, o, lse, cu, max(lengths), Hq, Hkv, 128,
                                               rope_pos=pos, rope_theta=1e6)
    assert torch.equal(fv, dv)
    assert _rel(fq, d[:, : Hq * 128]) < 1e-2 and _rel(fk, d[:, Hq * 128 : (Hq + Hkv) * 128]) < 1e-2
    assert (fq.float() - d[:, : Hq * 128].float()).abs().max() <= 2e-2 * d.float().abs().max()


@pytest.mark.parametrize("impl", [1, 2, 3])
@pytest.mark.parametrize("Hq,Hkv,splits", [(12, 2, 1), (32, 4, 4), (8, 8, 2), (16, 2, 3), (40, 2, 2), (4, 2, 1),
                                           (16, 4, 2)])
def test_paged_decode_and_cache_write(Hq, Hkv, splits, impl):
    """The three decode kernels (CUDA cores; tensor cores with the query heads, or the keys, as the
    MMA rows, both with TMA page gathers) against the fp32 reference, with lengths that leave empty
    splits and partial 128-token tiles; GQA groups 1, 2, 4, 6, 8 and 20 (16- and 32-wide transposed MMAs)."""
    if impl == 1 and Hq // Hkv not in (1, 2, 4, 6, 8):
        pytest.skip("the CUDA-core kernel is instantiated for GQA groups 1, 2, 4, 6 and 8")
    S, bs, D = 5, 16, 128
    lens = torch.tensor([1, 17, 300, 100, 129], dtype=torch.int32, device=DEV)
    max_blocks = 20
    nb = S * max_blocks
    kc = torch.zeros(nb, bs, Hkv, D, device=DEV, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    perm = torch.randperm(nb, device=DEV).to(torch.int32)
    table = perm.view(S, max_blocks)
    # write each sequence's K/V through the cache-write kernel
    for s in range(S):
        n = int(lens[s])
        kk = torch.randn(n, Hkv * D, device=DEV).bfloat16()
        vv = torch.randn(n, Hkv * D, device=DEV).bfloat16()
        t = torch.arange(n, device=DEV)
        slots = (table[s, t // bs].long() * bs + t % bs).to(torch.int32)
        ops.kv_cache_write(kk, vv, kc, vc, slots, Hkv)
        blocks = table[s, t // bs].long()
        assert torch.equal(kc[blocks, t % bs].reshape(n, -1), kk)
    q = torch.randn(S, Hq * D, device=DEV).bfloat16()
    out = ops.paged_decode(q, kc, vc, table, lens, Hq, Hkv, 1 / math.sqrt(D), num_splits=splits, impl=impl)
    want = ref.paged_decode(q.reshape(S, Hq, D), kc, vc, table, lens, 1 / math.sqrt(D))
    assert _rel(out, want.reshape(S, -1)) < 2e-2
    assert int(ops.status_tensor(torch.device(DEV))[0]) == 0


def test_sampler_greedy_and_distribution():
    rows, V = 6, 151936
    logits = (torch.randn(rows, V, device=DEV) * 2).bfloat16()
    temp = torch.zeros(rows, device=DEV)
    seeds = torch.arange(rows, device=DEV, dtype=torch.int64)
    offs = torch.zeros(rows, device=DEV, dtype=torch.int64)
    tok, lp = ops.sample(logits, temp, seeds, offs)
    assert torch.equal(tok, logits.float().argmax(-1))
    want = torch.log_softmax(logits.float(), -1).gather(1, tok.view(-1, 1)).squeeze(1)
    assert torch.allclose(lp, want, atol=2e-3)
    # temperature 1 on a 4-token support: empirical frequencies follow softmax
    small = torch.full((1, 64), -1e4, device=DEV)
    small[0, :4] = torch.tensor([0.0, 1.0, 2.0, 0.5], device=DEV)
    small = small.bfloat16().repeat(4000, 1)
    tok, lp = ops.sample(small, torch.ones(4000, device=DEV), torch.arange(4000, device=DEV), offs.new_zeros(4000),
                         num_chunks=1)
    freq = torch.bincount(tok, minlength=64)[:4].float() / 4000
    probs = torch.softmax(small[0, :4].float(), -1)
    assert torch.allclose(freq, probs, atol=0.03)


def _masked_logits(rows, V, seed=0):
    """Rows with -inf entries: whole leading chunks masked, scattered masks, and one row with a
    single finite logit."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = torch.randn(rows, V, generator=g) * 2
    x[0, : V // 2] = float("-inf")  # leading chunks entirely -inf
    x[1, torch.rand(V, generator=g) < 0.9] = float("-inf")
    x[2, :] = float("-inf")
    x[2, V - 3] = 1.5  # only one finite logit, in the last chunk
    x[3, 1::2] = float("-inf")
    return x.bfloat16().to(DEV)


@pytest.mark.parametrize("temp", [0.0, 1.0, 0.7])
def test_sampler_minus_inf_logits(temp):
    rows, V = 8, 151936
    logits = _masked_logits(rows, V)
    t = torch.full((rows,), temp, device=DEV)
    seeds = torch.arange(rows, device=DEV, dtype=torch.int64) + 11
    offs = torch.zeros(rows, device=DEV, dtype=torch.int64)
    tok, lp = ops.sample(logits, t, seeds, offs)
    assert torch.isfinite(lp).all(), lp
    assert torch.isfinite(logits.float().gather(1, tok.view(-1, 1))).all()  # never a masked token
    want = torch.log_softmax(logits.float(), -1).gather(1, tok.view(-1, 1)).squeeze(1)
    torch.testing.assert_close(lp, want, atol=2e-3, rtol=1e-4)
    assert int(tok[2]) == V - 3


def test_sampler_all_masked_row_has_no_nan():
    logits = torch.full((2, 4096), float("-inf"), device=DEV).bfloat16()
    logits[1, 7] = 0.0
    tok, lp = ops.sample(logits, torch.ones(2, device=DEV), torch.zeros(2, device=DEV, dtype=torch.int64),
                         torch.zeros(2, device=DEV, dtype=torch.int64))
    assert not torch.isnan(lp).any()
    assert int(tok[0]) == 0 and float(lp[0]) == float("-inf")
    assert int(tok[1]) == 7 and abs(float(lp[1])) < 1e-6


def _filtered_probs(x, temp, k, p):
    z = x.float() / temp
    if 0 < k < z.numel():
        z = z.masked_fill(z < torch.topk(z, k).values[-1], float("-inf"))
    probs = torch.softmax(z, -1)
    if p < 1:
        sp, order = torch.sort(probs, descending=True)
        keep = (torch.cumsum(sp, 0) - sp) < p
        probs = torch.zeros_like(probs).scatter_(0, order, sp * keep)
        probs = probs / probs.sum()
    return probs


@pytest.mark.parametrize("k,p", [(5, 1.0), (0, 0.8), (6, 0.7), (1, 1.0), (0, 0.05)])
def test_sampler_top_k_top_p_distribution(k, p):
    V, n = 4096, 20000
    base = torch.full((V,), -6.0)
    base[:12] = torch.tensor([2.0, 1.6, 1.5, 1.2, 1.0, 0.9, 0.5, 0.3, 0.2, 0.0, -0.5, -1.0])
    base = base.bfloat16()
    logits = base.to(DEV).repeat(n, 1)
    temp = 0.9
    tok, lp = ops.sample(logits, torch.full((n,), temp, device=DEV), torch.arange(n, device=DEV),
                         torch.full((n,), 3, device=DEV, dtype=torch.int64),
                         top_k=torch.full((n,), k, dtype=torch.int32), top_p=torch.full((n,), p))
    want = _filtered_probs(base, temp, k, p)
    freq = torch.bincount(tok.cpu(), minlength=V).float() / n
    assert float(freq[want == 0].sum()) == 0.0  # nothing outside the kept set
    assert torch.allclose(freq, want, atol=0.015), (freq[:12], want[:12])
    full = torch.log_softmax(base.float(), -1)
    torch.testing.assert_close(lp.cpu(), full[tok.cpu()], atol=2e-3, rtol=1e-4)


def test_sampler_mixed_rows_filtered_and_plain():
    """Rows with and without filters in one call: plain rows equal a call without filter arrays."""
    rows, V = 64, 151936
    logits = (torch.randn(rows, V, device=DEV) * 3).bfloat16()
    t = torch.rand(rows, device=DEV) + 0.5
    t[::9] = 0.0
    seeds = torch.randint(0, 2**62, (rows,), device=DEV)
    offs = torch.arange(rows, device=DEV, dtype=torch.int64)
    top_k = torch.zeros(rows, dtype=torch.int32)
    top_p = torch.ones(rows)
    top_k[1::4] = 20
    top_p[2::4] = 0.5
    tok, lp = ops.sample(logits, t, seeds, offs, top_k=top_k, top_p=top_p)
    tok0, lp0 = ops.sample(logits, t, seeds, offs)
    plain = ((top_k == 0) & (top_p == 1.0)) | (t.cpu() <= 0)
    assert torch.equal(tok[plain.to(DEV)], tok0[plain.to(DEV)])
    for i in torch.nonzero(top_k > 0).flatten().tolist():
        if float(t[i]) > 0:
            kth = torch.topk(logits[i].float(), 20).values[-1]
            assert float(logits[i, tok[i]].float()) >= float(kth)
    want = torch.log_softmax(logits.float(), -1).gather(1, tok.view(-1, 1)).squeeze(1)
    torch.testing.assert_close(lp, want, atol=2e-3, rtol=1e-4)


@pytest.mark.parametrize("splits", [2, 4, 0])
def test_gemm_split_k_accumulate(splits):
    M, N, K = 256, 512, 4096
    A = torch.randn(M, K, device=DEV).bfloat16()
    B = torch.randn(N, K, device=DEV).bfloat16()
    acc = torch.randn(M, N, device=DEV)
    base = acc.clone()
    ops.gemm(A.t().contiguous(), B.t().contiguous(), acc, a_mn=True, b_mn=True, beta=1.0, out_dtype=torch.float32,
             splits=splits)
    assert _rel(acc, base + A.float() @ B.float().t()) < 1e-5


@pytest.mark.parametrize("M", [1, 7, 64, 256])
def test_skinny_linear_split_k_with_bias_residual(M):
    N, K = 2048, 1536
    x = torch.randn(M, K, device=DEV).bfloat16()
    w = (torch.randn(N, K, device=DEV) * 0.05).bfloat16()
    b = torch.randn(N, device=DEV).bfloat16()
    r = torch.randn(M, N, device=DEV).bfloat16()
    y = ops.linear(x, w, bias=b, residual=r)
    assert _rel(y, x.float() @ w.float().t() + b.float() + r.float()) < 1e-2


@pytest.mark.parametrize("q_lens,k_lens", [([5, 130, 1], [300, 130, 77]), ([200], [1000])])
def test_attention_forward_queries_over_longer_keys(q_lens, k_lens):
    Hq, Hkv, D = 4, 2, 128
    cu_q = torch.tensor([0] + list(torch.tensor(q_lens).cumsum(0)), dtype=torch.int32, device=DEV)
    cu_k = torch.tensor([0] + list(torch.tensor(k_lens).cumsum(0)), dtype=torch.int32, device=DEV)
    q = torch.randn(sum(q_lens), Hq * D, device=DEV).bfloat16()
    k = torch.randn(sum(k_lens), Hkv * D, device=DEV).bfloat16()
    v = torch.randn(sum(k_lens), Hkv * D, device=DEV).bfloat16()
    o, lse = ops.attention_varlen(q, k, v, cu_q, max(q_lens), Hq, Hkv, D, cu_seqlens_k=cu_k)
    o_r, lse_r = ref.attention_varlen_qk(q.reshape(-1, Hq, D), k.reshape(-1, Hkv, D), v.reshape(-1, Hkv, D), cu_q,
                                         cu_k, 1 / math.sqrt(D))
    assert _rel(o, o_r.reshape(o.shape)) < 2e-2
    assert torch.allclose(lse, lse_r, atol=1e-2)


def test_grouped_expert_gemms_match_per_expert_products():
    from accerl_agent_b200.models.moe import _grouped, padded_layout

    E, H, N = 5, 256, 384
    counts = [0, 130, 7, 256, 1]
    lay = padded_layout(counts, torch.device(DEV))
    R = lay["total"]
    x = torch.zeros(R, H, device=DEV).bfloat16()
    dy = torch.zeros(R, N, device=DEV).bfloat16()
    for e, c in enumerate(counts):
        s = lay["starts"][e]
        x[s : s + c] = torch.randn(c, H, device=DEV).bfloat16()
        dy[s : s + c] = torch.randn(c, N, device=DEV).bfloat16()
    W = (torch.randn(E, N, H, device=DEV) * 0.05).bfloat16()
    y = torch.empty(R, N, device=DEV).bfloat16()
    _grouped(x, False, W.view(E * N, H), False, y, R, N, H, 1, lay, N)  # forward  y_e = x_e W_e^T
    dx = torch.empty(R, H, device=DEV).bfloat16()
    _grouped(dy, False, W.view(E * N, H), True, dx, R, H, N, 1, lay, N)  # dgrad    dx_e = dy_e W_e
    gW = torch.ones(E * N, H, device=DEV)
    _grouped(dy, True, x, True, gW, N, H, R, 2, lay, 0, N, beta=1.0)  # wgrad  gW_e += dy_e^T x_e
    for e, c in enumerate(counts):
        s = lay["starts"][e]
        xe, dye, We = x[s : s + c].float(), dy[s : s + c].float(), W[e].float()
        if c:
            assert _rel(y[s : s + c], xe @ We.t()) < 1e-2
            assert _rel(dx[s : s + c], dye @ We) < 1e-2
        assert _rel(gW[e * N : (e + 1) * N], 1.0 + dye.t() @ xe) < 1e-5


def test_moe_combine_fwd_bwd():
    T, k, H, R = 300, 4, 2048, 1600
    ys = torch.randn(R, H, device=DEV).bfloat16()
    pos = torch.randperm(R, device=DEV)[: T * k]
    w = torch.rand(T * k, device=DEV)
    res = torch.randn(T, H, device=DEV).bfloat16()
    sh = torch.randn(T, H, device=DEV).bfloat16()
    sg = torch.rand(T, 1, device=DEV)
    out = ops.moe_combine(ys, pos, w, k, residual=res, shared=sh, sg=sg)
    ref = res.float() + (ys.float()[pos] * w[:, None]).view(T, k, H).sum(1) + sg * sh.float()
    assert _rel(out, ref) < 1e-2
    dout = torch.randn(T, H, device=DEV).bfloat16()
    dys = torch.zeros(R, H, device=DEV, dtype=torch.bfloat16)
    dw = ops.moe_combine_backward(dout, ys, pos, w, k, dys)
    g = dout.float().repeat_interleave(k, 0)
    assert _rel(dw, (g * ys.float()[pos]).sum(-1)) < 1e-3
    assert _rel(dys[pos], g * w[:, None]) < 1e-2
    untouched = torch.ones(R, dtype=torch.bool, device=DEV)
    untouched[pos] = False
    assert bool((dys[untouched] == 0).all())


@pytest.mark.parametrize("E,k,norm", [(60, 4, False), (128, 8, True), (8, 2, False)])
def test_moe_router_kernel(E, k, norm):
    """Fused router (tcgen05 logits GEMM with a ragged expert count + softmax / top-k / renorm / counts
    kernel) against the PyTorch router on the same bf16 logits."""
    from types import SimpleNamespace

    from accerl_agent_b200.models import moe

    T, H = 1000, 512
    h = torch.randn(T, H, device=DEV).bfloat16()
    W = (torch.randn(E, H, device=DEV) * 0.05).bfloat16()
    cfg = SimpleNamespace(num_experts=E, num_experts_per_tok=k, norm_topk_prob=norm)
    model = SimpleNamespace(cfg=cfg, w=lambda name: W)
    probs, topw, topi, cnt = moe.route(model, 0, h, counts=True)
    # logits rounded to bf16 from fp32 sums in a different order can differ by one bf16 step
    logits = (h.float() @ W.float().t()).bfloat16().float()
    want_p = torch.softmax(logits, -1)
    assert torch.allclose(probs, want_p, atol=1e-4, rtol=2e-2)
    assert torch.allclose(probs.sum(-1), torch.ones(T, device=DEV), atol=1e-5)
    # bf16 logits tie often; compare the chosen weights as sorted multisets and require every chosen
    # expert to be within the top k of the kernel's own probabilities
    want_w, _ = want_p.topk(k, -1)
    if norm:
        want_w = want_w / want_w.sum(-1, keepdim=True)
    assert torch.allclose(topw.sort(-1).values, want_w.sort(-1).values, atol=1e-4, rtol=2e-2)
    kth = probs.topk(k, -1).values[:, -1:]
    assert bool((probs.gather(1, topi) >= kth).all())
    assert bool((topi.sort(-1).values[:, 1:] != topi.sort(-1).values[:, :-1]).all())  # distinct experts
    # the kernel's own weights are consistent with its probabilities
    sel = probs.gather(1, topi)
    if norm:
        sel = sel / sel.sum(-1, keepdim=True)
    assert torch.allclose(topw, sel, atol=1e-6, rtol=1e-5)
    assert torch.equal(cnt.long(), torch.bincount(topi.reshape(-1), minlength=E))


@pytest.mark.parametrize("T,E,k,lo,El,skew", [(1000, 60, 4, 0, 60, False), (4099, 128, 8, 0, 128, True),
                                                (2500, 64, 2, 16, 24, False), (3, 8, 2, 0, 8, False)])
def test_moe_dispatch_kernel(T, E, k, lo, El, skew):
    """One-pass dispatch (``moe_layout`` kernels) against the torch formulation of the same layout:
    identical rows for every (token, slot) pair (stable within an expert), tile map, segment starts and
    sizes, counts; weights rounded to bf16 (0 outside the shard's range); xs rows equal their token's
    hidden row and padding rows are zero."""
    from accerl_agent_b200.models.moe import device_dispatch, device_padded_layout

    g = torch.Generator().manual_seed(T)
    if skew:  # most pairs on a few experts: segments much longer than one 1024-pair block
        scores = torch.rand(T, E, generator=g) + (torch.arange(E) < 3).float() * 2
    else:
        scores = torch.rand(T, E, generator=g)
    topi = scores.topk(k, -1).indices.to(DEV)
    topw = torch.rand(T, k, generator=g).to(DEV)
    H = 256
    h = torch.randn(T, H, device=DEV).bfloat16()
    for _ in range(2):  # the histogram scratch keeps the last call's contents
        xs, pos, w, lay = device_dispatch(topi, topw, h, E, lo, El, zero_pad=True)
        torch.cuda.synchronize()
        order, rows, valid, ref = device_padded_layout(topi, E, lo, El)
        assert lay["total"] == ref["total"]
        want_pos = torch.empty_like(pos)
        want_pos[order] = rows
        assert torch.equal(pos, want_pos)
        for key in ("tile_expert", "row_start", "rows"):
            assert torch.equal(lay[key], ref[key].to(torch.int32)), key
        assert torch.equal(lay["counts"].long(), torch.bincount(topi.reshape(-1), minlength=E))
        ok = pos < lay["total"]
        want_w = torch.where(ok, topw.reshape(-1).bfloat16().float(), torch.zeros_like(w))
        assert torch.equal(w, want_w)
        tok = torch.arange(T * k, device=DEV) // k
        assert torch.equal(xs[pos[ok]], h[tok[ok]])
        used = torch.zeros(lay["total"], dtype=torch.bool, device=DEV)
        used[pos[ok]] = True
        assert bool((xs[~used] == 0).all())


@pytest.mark.parametrize("Hq,Hkv,qk_norm", [(6, 2, False), (16, 4, True), (7, 1, True)])
def test_qkv_rope_cache_fused(Hq, Hkv, qk_norm):
    """The engine's fused post-projection kernel (qk-norm, RoPE, paged cache write) against the
    separate kernels it replaces, run in the same order; rows with slot -1 leave the caches alone."""
    T, D, blocks, bs = 300, 128, 64, 16
    qkv = torch.randn(T, (Hq + 2 * Hkv) * D, device=DEV).bfloat16()
    pos = torch.randint(0, 30000, (T,), device=DEV)
    slots = torch.randperm(blocks * bs, device=DEV)[:T].to(torch.int32)
    slots[::7] = -1
    qn = (1 + 0.1 * torch.randn(D, device=DEV)).bfloat16() if qk_norm else None
    kn = (1 + 0.1 * torch.randn(D, device=DEV)).bfloat16() if qk_norm else None
    kc = torch.full((blocks, bs, Hkv, D), 7.0, device=DEV).bfloat16()
    vc = kc.clone()
    want_qkv, want_kc, want_vc = qkv.clone(), kc.clone(), vc.clone()
    qd, kd = Hq * D, Hkv * D
    if qk_norm:
        a, _ = ops.rmsnorm(want_qkv[:, :qd].reshape(T * Hq, D).clone(), qn, 1e-6)
        b, _ = ops.rmsnorm(want_qkv[:, qd : qd + kd].reshape(T * Hkv, D).clone(), kn, 1e-6)
        want_qkv[:, :qd].copy_(a.view(T, qd))
        want_qkv[:, qd : qd + kd].copy_(b.view(T, kd))
    ops.rope_(want_qkv, pos, Hq + Hkv, D, 1e6)
    ops.kv_cache_write(want_qkv[:, qd : qd + kd], want_qkv[:, qd + kd :], want_kc, want_vc, slots, Hkv)
    got = qkv.clone()
    ops.native().qkv_rope_cache(got, pos, slots, kc, vc, Hq, Hkv, 1e6, qn, kn, 1e-6)
    torch.cuda.synchronize()
    for g, w in ((got, want_qkv), (kc, want_kc), (vc, want_vc)):
        # same roundings in the same order; a contraction of a*b - c*d into an FMA may differ by one
        # bf16 step on rare elements
        torch.testing.assert_close(g.float(), w.float(), atol=1e-6, rtol=2 ** -7)
        assert (g != w).float().mean().item() < 1e-3
    untouched = torch.ones(blocks * bs, dtype=torch.bool, device=DEV)
    untouched[slots[slots >= 0].long()] = False
    assert bool((kc.view(-1, Hkv, D)[untouched] == 7.0).all()) and bool((vc.view(-1, Hkv, D)[untouched] == 7.0).all())


@pytest.mark.parametrize("block_n", [0, 256, 128, -256])
def test_gemm_rope_epilogue(block_n):
    """qkv projection with the rotary embedding in the epilogue equals the projection followed by the
    RoPE kernel (q and k heads rotated, v heads untouched), with bias and a row tail."""
    T, H, Hq, Hkv, D = 777, 384, 6, 2, 128
    x = torch.randn(T, H, device=DEV).bfloat16()
    w = (torch.randn((Hq + 2 * Hkv) * D, H, device=DEV) * 0.05).bfloat16()
    bias = torch.randn((Hq + 2 * Hkv) * D, device=DEV).bfloat16()
    pos = torch.randint(0, 8192, (T,), device=DEV)
    want = ops.gemm(x, w, bias=bias)
    ops.rope_(want, pos, Hq + Hkv, D, 1e6)
    got = torch.empty_like(want)
    ops.native().gemm_rope(x, w, got, bias, pos, (Hq + Hkv) * D, 1e6, ops.status_tensor(torch.device(DEV)), block_n, 0)
    # identical up to fp32 contraction differences in the rotation
    assert (got.float() - want.float()).abs().max() <= 1e-2 * want.float().abs().max()
    assert torch.equal(got[:, (Hq + Hkv) * D :], want[:, (Hq + Hkv) * D :])  # v
    got2 = ops.linear_rope(x, w, bias, pos, Hq + Hkv, D, 1e6)
    assert torch.equal(got2, got) or block_n != 0


@pytest.mark.parametrize("n,V,chunk", [(300, 151936, 16384), (64, 4096, 1024), (7, 1000, 256)])
def test_lm_head_chunked_matches_fp32_oracle(n, V, chunk):
    """Vocabulary-chunked response-only LM head (logprob, lse, entropy; d(rows), d(W)) against fp32
    autograd over the full logits."""
    H = 256
    g = torch.Generator(device="cpu").manual_seed(n)
    rows = (torch.randn(n, H, generator=g) * 0.5).bfloat16().to(DEV)
    W = (torch.randn(V, H, generator=g) * 0.05).bfloat16().to(DEV)
    labels = torch.randint(0, V, (n,), generator=g).to(DEV)
    grad = torch.randn(n, generator=g).to(DEV)
    lp, lse, ent = ops.lm_head_logprobs(rows, W, labels, with_entropy=True, chunk=chunk)
    gW = torch.zeros(V, H, device=DEV)
    drows = ops.lm_head_backward(rows, W, labels, lse, grad, gW, True, chunk=chunk)
    x = rows.float().requires_grad_(True)
    w = W.float().requires_grad_(True)
    logp = torch.log_softmax(x @ w.t(), -1)
    lp_ref = logp.gather(1, labels.view(-1, 1)).squeeze(1)
    ent_ref = -(logp.exp() * logp).sum(-1)
    (lp_ref * grad).sum().backward()
    torch.testing.assert_close(lp, lp_ref.detach(), atol=2e-2, rtol=2e-3)
    torch.testing.assert_close(ent, ent_ref.detach(), atol=2e-2, rtol=2e-3)
    assert _rel(drows.float(), x.grad) < 2e-2
    assert _rel(gW, w.grad) < 2e-2


def test_lm_head_never_builds_full_logits():
    n, H, V = 2048, 1536, 151936
    rows = torch.randn(n, H, device=DEV).bfloat16()
    W = (torch.randn(V, H, device=DEV) * 0.02).bfloat16()
    labels = torch.randint(0, V, (n,), device=DEV)
    ops.lm_head_logprobs(rows, W, labels)  # workspaces allocated once
    torch.cuda.synchronize()
    base = torch.cuda.memory_allocated()
    torch.cuda.reset_peak_memory_stats()
    lp, lse, _ = ops.lm_head_logprobs(rows, W, labels)
    gW = torch.zeros(V, H, device=DEV)
    torch.cuda.synchronize()
    base2 = torch.cuda.memory_allocated()
    torch.cuda.reset_peak_memory_stats()
    ops.lm_head_backward(rows, W, labels, lse, torch.ones(n, device=DEV), gW)
    torch.cuda.synchronize()
    full_logits = n * V * 2  # 622 MB
    assert torch.cuda.max_memory_allocated() - base2 < full_logits // 4
    assert torch.isfinite(lp).all()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_native_ops_follow_their_tensors_device_from_any_thread():
    """The CUDA current device is per thread: a thread that never selected a device (current device
    0) still launches the native kernels of cuda:1 tensors on cuda:1."""
    import threading

    dev = torch.device("cuda", 1)
    x = torch.randn(64, 256, device=dev).bfloat16()
    w = (torch.rand(256, device=dev) + 0.5).bfloat16()
    W = (torch.randn(128, 256, device=dev) * 0.05).bfloat16()
    out = {}

    def run():
        out["device"] = torch.cuda.current_device()
        y, _ = ops.rmsnorm(x, w, 1e-6)
        out["y"] = y
        out["z"] = ops.linear(y, W)
        torch.cuda.synchronize(dev)

    t = threading.Thread(target=run)
    t.start()
    t.join()
    assert out["device"] == 0
    want = ref.rmsnorm(x.float().cpu(), w.float().cpu(), 1e-6)[0]
    assert _rel(out["y"].float().cpu(), want) < 2e-2
    assert _rel(out["z"].float().cpu(), want @ W.float().cpu().t()) < 3e-2
