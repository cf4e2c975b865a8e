"""GPU parity of the FP8 target and W4 draft lm_heads.

FP8: the fused prologue's quantized activation is bit-exact to per_token_group_quant_fp8;
logits against the fp32 oracle ``(qx*xs) @ (wq*ws)^T`` (tests/k3/test_fp8sk.py:69,77) with
the reference's own acceptance bound ``max|y-ref|/max|ref| < 3*3.7e-3 + 1e-4``; the fp32 row
statistics (max within 1e-5, logsumexp within 1e-4 absolute, argmax exact except on at most
one row per call whose oracle top-2 gap is at most 1e-4, with the count printed); max
|dlogit| and |dlogprob| printed. W4: against
``F.linear(x.half().float(), unpack_w4(p))`` with the reference's rel-Frobenius < 5e-3
(tests/k3/w4_verify.py:35-56) over M in {1,2,3,5,16,20,64,129} and N=1000 padding.
Both at the full head shape N=151936, K=2560 too. Graph replay == eager."""
from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from conftest import load_pkg
from oracle import quant_oracle as Q

pytestmark = pytest.mark.gpu
P = load_pkg()
F8 = P.fp8_target_lmhead
W4 = P.draft_w4_lmhead
FP8 = torch.float8_e4m3fn
REL_FP8 = 3 * 3.7e-3 + 1e-4          # tests/k3/test_fp8sk.py:95 with the measured 3.7e-3


def _fp8_weight(N, K, seed, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    w = (torch.randn(N, K, device=dev, generator=g) * 0.02).bfloat16()
    wq, ws = F8.pack_fp8_block(w)
    wrow = F8.unpack_fp8_block(wq)
    return wq, ws, Q.dequant_fp8_block(wrow, ws)


# argmax: exact, except on rows whose oracle top-2 gap is at most ARGMAX_GAP (the kernel's
# fp32 sums run in another order than the oracle's matmul, a few 1e-6 apart); at most
# ARGMAX_MAX_EXEMPT such rows per call are tolerated, and their number is printed
ARGMAX_GAP = 1e-4
ARGMAX_MAX_EXEMPT = 1


def _check_stats(tag, logits_ref, mx, arg, lse, offset=0):
    rmx, rarg, rlse = Q.row_stats(logits_ref)
    gap = Q.top2_gap(logits_ref)
    assert torch.allclose(mx.cpu(), rmx.cpu(), rtol=1e-5, atol=1e-5), tag
    assert (lse.cpu() - rlse.cpu()).abs().max().item() < 1e-4, tag
    exempt = [m for m in range(mx.numel()) if gap[m] <= ARGMAX_GAP]
    for m in range(mx.numel()):
        if m not in exempt:
            assert int(arg[m]) == int(rarg[m]) + offset, f"{tag} row {m}"
    print(f"{tag}: argmax exempt rows {len(exempt)}/{mx.numel()} (top-2 gap <= {ARGMAX_GAP}), "
          f"max|dmax| {(mx.cpu() - rmx.cpu()).abs().max().item():.2e}, "
          f"max|dlse| {(lse.cpu() - rlse.cpu()).abs().max().item():.2e}")
    assert len(exempt) <= ARGMAX_MAX_EXEMPT, (tag, exempt)
    lp = (logits_ref.double() - rlse.double().unsqueeze(1).to(logits_ref.device))
    return lp


@pytest.mark.parametrize("M", [1, 2, 3, 5, 8, 9, 12, 16, 20, 33, 64])
def test_fp8_fused_small_shape(cuda, M):
    N, K = 8192, 2560
    wq, ws, wdq = _fp8_weight(N, K, N * 7 + K, cuda)
    g = torch.Generator(device=cuda).manual_seed(M * 13 + N)
    x = torch.randn(M, K, device=cuda, dtype=torch.bfloat16, generator=g)
    y, mx, arg, lse, qx, xs = F8.fp8_lmhead(x, wq, ws, debug_quant=True)
    rq, rs = Q.group_quant_fp8(x, 128)
    assert torch.equal(qx.view(torch.uint8), rq.view(torch.uint8)) and torch.equal(xs, rs)
    ref = Q.fp8_block_gemm_ref(rq, rs, wdq)
    rel = ((y.float() - ref).abs().max() / ref.abs().max().clamp(min=1e-9)).item()
    assert rel < REL_FP8, rel
    _check_stats(f"M={M}", ref, mx, arg, lse)
    # the plain GEMM entry gives the same logits
    assert torch.equal(F8.gemm_fp8_block(x, wq, ws), y)


def test_fp8_prequantized_abi(cuda):
    N, K, M = 2560, 3072, 5
    wq, ws, wdq = _fp8_weight(N, K, 1, cuda)
    x = torch.randn(M, K, device=cuda, dtype=torch.bfloat16)
    qx, xs = P.fused_silu_mul_quant.per_token_group_quant_fp8(x, 128)
    y = F8.fp8_block_scaled_mm(qx, wq, xs, ws)
    ref = Q.fp8_block_gemm_ref(qx, xs, wdq)
    assert ((y.float() - ref).abs().max() / ref.abs().max()).item() < REL_FP8
    # hcq entry, legal knobs, same result
    lib = P._lib.lmhead()
    y2 = torch.empty_like(y)
    rc = lib.hcq_gemm_fp8blk_nt_m16(P._lib.ptr(qx), P._lib.ptr(xs), P._lib.ptr(wq), P._lib.ptr(ws),
                                    P._lib.ptr(y2), M, K, N, 2, 4, 1, P._lib.stream_ptr())
    assert rc == 0 and torch.equal(y, y2)


@pytest.mark.parametrize("M", [1, 5, 16, 20, 64])
def test_fp8_fused_baseline_shape(cuda, M):
    """Full target head: W ~N(0,0.02) [151936, 2560], x ~N(0,1). At this size every CTA streams
    many strips, so the ring's slots turn over many times; the device error word (a pipeline
    wait that ran out) must stay clear."""
    N, K = 151936, 2560
    wq, ws, wdq = _fp8_weight(N, K, 0, cuda)
    x = torch.randn(M, K, device=cuda, dtype=torch.bfloat16, generator=torch.Generator(device=cuda).manual_seed(M))
    y, mx, arg, lse = F8.fp8_lmhead(x, wq, ws)
    rq, rs = Q.group_quant_fp8(x, 128)
    ref = Q.fp8_block_gemm_ref(rq, rs, wdq)
    d = (y.float() - ref).abs()
    rel = (d.max() / ref.abs().max()).item()
    lp = _check_stats(f"N={N} M={M}", ref, mx, arg, lse)
    dlp = ((y.float() - lse.unsqueeze(1)) - lp.float()).abs().max().item()
    print(f"FP8 N={N} M={M}: rel {rel:.3e}, max|dlogit| {d.max().item():.3e}, max|dlogprob| {dlp:.3e}")
    assert rel < REL_FP8
    assert P._lib.lmhead().b200_lmhead_error(1) == 0
    del wdq, ref


def test_fp8_vocab_shards_combine(cuda):
    """Shard on 128-row blocks with vocab_offset: the combined (max, argmax, lse) equals the
    unsharded call's."""
    N, K, M = 128 * 37, 2560, 4
    wq, ws, wdq = _fp8_weight(N, K, 5, cuda)
    x = torch.randn(M, K, device=cuda, dtype=torch.bfloat16)
    _, mx, arg, lse = F8.fp8_lmhead(x, wq, ws, want_logits=False)
    parts = []
    for r0, r1 in P.sharded.vocab_shards(N, 3):
        _, m_, a_, l_ = F8.fp8_lmhead(x, wq[r0:r1], ws[r0 // 128:r1 // 128], vocab_offset=r0, want_logits=False)
        parts.append((m_, a_, l_))
    cm, ca, cl = P.sharded.combine_row_stats_local(parts)
    assert torch.equal(ca, arg) and torch.allclose(cm, mx) and torch.allclose(cl, lse, atol=1e-5)


def test_combine_kernels_match_reference(cuda):
    """b200_pack_row_stats + b200_combine_row_stats (the CUDA side of combine_row_stats) give
    the torch combine's result on the same gathered triples, ties going to the first rank."""
    L = P._lib
    lib = L.lmhead()
    W, M = 3, 37
    g = torch.Generator(device=cuda).manual_seed(5)
    mx = torch.randn(W, M, device=cuda, generator=g)
    mx[1, :5] = mx[0, :5]
    mx[2, 5:9] = mx[1, 5:9]
    arg = torch.randint(0, 1 << 20, (W, M), device=cuda, generator=g, dtype=torch.int64)
    lse = mx + torch.rand(W, M, device=cuda, generator=g)
    packed = torch.empty(W, M, 3, dtype=torch.float64, device=cuda)
    for r in range(W):
        assert lib.b200_pack_row_stats(L.ptr(mx[r]), L.ptr(arg[r]), L.ptr(lse[r]), M, L.ptr(packed[r]),
                                       L.stream_ptr()) == 0
    gm = torch.empty(M, device=cuda)
    ga = torch.empty(M, dtype=torch.int64, device=cuda)
    gl = torch.empty(M, device=cuda)
    assert lib.b200_combine_row_stats(L.ptr(packed), W, M, L.ptr(gm), L.ptr(ga), L.ptr(gl), L.stream_ptr()) == 0
    rm, ra, rl = P.sharded._combine(packed[:, :, 0], packed[:, :, 1].to(torch.int64), packed[:, :, 2])
    assert torch.equal(ga, ra) and torch.equal(gm, rm) and torch.allclose(gl, rl, atol=1e-6)


def test_fp8_graph_replay(cuda):
    N, K, M = 4096, 2560, 5
    wq, ws, _ = _fp8_weight(N, K, 2, cuda)
    x = torch.randn(M, K, device=cuda, dtype=torch.bfloat16)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):
            F8.fp8_lmhead(x, wq, ws)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        yg, mg, ag, lg = F8.fp8_lmhead(x, wq, ws)
    for _ in range(3):
        x.copy_(torch.randn(M, K, device=cuda, dtype=torch.bfloat16))
        g.replay()
        y, mx, arg, lse = F8.fp8_lmhead(x, wq, ws)
        torch.cuda.synchronize()
        assert torch.equal(yg, y) and torch.equal(ag, arg) and torch.equal(mg, mx) and torch.equal(lg, lse)
    assert P._lib.lmhead().b200_lmhead_error(1) == 0


# ---------------------------------------------------------------------------------------
# W4
# ---------------------------------------------------------------------------------------

def _rel(y, r):
    return ((y.float() - r).norm() / r.norm()).item()


def test_w4_pack_on_gpu_round_trip(cuda):
    """unpack_w4 == dequant(quantize_w4) exactly (tests/k3/w4_verify.py:22-32), GPU packing."""
    for n, k in [(256, 512), (1024, 2560), (48, 128), (1000, 256)]:
        w = (torch.randn(n, k, device=cuda) * 0.02).bfloat16()
        p = W4.pack_w4a16(w)
        q, s, z = W4.quantize_w4(w.float())
        ref = Q.w4_dequant(q, s, z)
        got = W4.unpack_w4(p, torch.float32)[:n]
        assert torch.equal(got, ref)


@pytest.mark.parametrize("M", [1, 2, 3, 4, 5, 16, 20, 64, 129])
def test_w4_gemm_vs_dequant_reference(cuda, M):
    n, k = 1024, 2560
    torch.manual_seed(0)
    w = (torch.randn(n, k, device=cuda) * 0.02).bfloat16()
    p = W4.pack_w4a16(w)
    wref = W4.unpack_w4(p, torch.float32)
    x = torch.randn(M, k, device=cuda).bfloat16()
    y = W4.gemm_w4a16(x, p)
    r = F.linear(x.float().half().float(), wref)
    assert y.shape == (M, n) and _rel(y, r) < 5e-3
    assert ((y.float() - r).abs().max() / r.abs().max()).item() < 4e-3


def test_w4_padding_and_top(cuda):
    n2, k = 1000, 2560
    w2 = (torch.randn(n2, k, device=cuda) * 0.02).bfloat16()
    w2[997] = 0.5                                           # a winning row near the padding edge
    p2 = W4.pack_w4a16(w2)
    x = torch.randn(5, k, device=cuda).bfloat16().abs()
    y = W4.gemm_w4a16(x, p2)
    wref = W4.unpack_w4(p2, torch.float32)[:n2]
    r = F.linear(x.float().half().float(), wref)
    assert y.shape == (5, n2) and _rel(y, r) < 5e-3
    logits, mx, arg, lse = W4.gemm_w4a16_top(x, p2, vocab_offset=1000)
    assert torch.equal(logits, y)
    rmx, rarg, rlse = Q.row_stats(r)
    assert torch.equal(arg.cpu(), rarg.cpu().long() + 1000)
    assert (lse.cpu() - rlse.cpu()).abs().max().item() < 1e-3


@pytest.mark.parametrize("M", [1, 4, 16])
def test_w4_sym_format(cuda, M):
    """Symmetric int4 with bf16 group scales (b200_w4_lmhead_sym): logits against
    F.linear(f16(x), dequant) within the reference's rel-Frobenius 5e-3, the opaque op and the
    fused top-k path agree, argmax exact where the top-2 gap allows, padding never wins."""
    n, k = 1000, 2560
    g = torch.Generator(device=cuda).manual_seed(M)
    w = (torch.randn(n, k, device=cuda, generator=g) * 0.02).bfloat16()
    w[996] = 0.4
    p = W4.pack_w4a16_sym(w)
    x = torch.randn(M, k, device=cuda, generator=g).bfloat16()
    x[0] = x[0].abs()
    y = W4.gemm_w4a16(x, p)
    wref = W4.unpack_w4(p, torch.float32)[:n]
    r = F.linear(x.float().half().float(), wref)
    assert y.shape == (M, n) and _rel(y, r) < 5e-3
    logits, mx, arg, lse = W4.gemm_w4a16_top(x, p, vocab_offset=7)
    assert torch.equal(logits, y)
    rmx, rarg, rlse = Q.row_stats(r)
    gap = Q.top2_gap(r)
    for m in range(M):
        if gap[m] > 1e-3:
            assert int(arg[m]) == int(rarg[m]) + 7
    assert (lse.cpu() - rlse.cpu()).abs().max().item() < 1e-3
    assert P._lib.lmhead().b200_lmhead_error(1) == 0


def test_w4_reference_c_abi_f16(cuda):
    """r4d_gemm_w4a16_nt_m64 with an f16 activation (the reference's call, draft_w4_lmhead.py:363-369)."""
    n, k, M = 512, 2560, 5
    w = (torch.randn(n, k, device=cuda) * 0.02).bfloat16()
    p = W4.pack_w4a16(w)
    x = torch.randn(M, k, device=cuda).bfloat16()
    a = x.to(torch.float16).contiguous()
    c = torch.empty(M, p.n_pad, dtype=torch.bfloat16, device=cuda)
    lib = P._lib.lmhead()
    lib.r4d_gemm_w4a16_nt_m64(a.data_ptr(), p.wq.data_ptr(), p.wsz.data_ptr(), c.data_ptr(),
                              M, k, p.n_pad, 1, 10, 1, 1, 1, torch.cuda.current_stream().cuda_stream)
    assert lib.r4d_gemm_w4a16_nt_m64_last_error() == 0
    assert torch.equal(c, W4.gemm_w4a16(x, p))


@pytest.mark.parametrize("M,sym", [(4, False), (16, False), (4, True)])
def test_w4_baseline_shape(cuda, M, sym):
    """Full draft head: x [M, 2560] ~N(0,1), W ~N(0,0.02) [151936, 2560]; M=16 takes the wider
    activation region (fewer ring stages); the device error word must stay clear."""
    n, k = 151936, 2560
    w = (torch.randn(n, k, device=cuda, generator=torch.Generator(device=cuda).manual_seed(0)) * 0.02).bfloat16()
    p = W4.pack_w4a16_sym(w) if sym else W4.pack_w4a16(w)
    del w
    x = torch.randn(M, k, device=cuda, generator=torch.Generator(device=cuda).manual_seed(1)).bfloat16()
    logits, mx, arg, lse = W4.gemm_w4a16_top(x, p)
    wref = W4.unpack_w4(p, torch.float32)[:n]
    r = F.linear(x.float().half().float(), wref)
    del wref
    rel = _rel(logits, r)
    rmx, rarg, rlse = Q.row_stats(r)
    gap = Q.top2_gap(r)
    print(f"W4 N={n} M={M}: rel-Frobenius {rel:.3e}, top2 gaps {gap.tolist()}")
    assert rel < 5e-3
    assert P._lib.lmhead().b200_lmhead_error(1) == 0
    for m in range(M):
        if gap[m] > 1e-3:
            assert int(arg[m]) == int(rarg[m])


def test_w4_graph_replay(cuda):
    n, k = 2048, 2560
    p = W4.pack_w4a16((torch.randn(n, k, device=cuda) * 0.02).bfloat16())
    x = torch.randn(5, k, device=cuda).bfloat16()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(3):
            W4.gemm_w4a16(x, p)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        yg = W4.gemm_w4a16(x, p)
    x.copy_(torch.randn(5, k, device=cuda).bfloat16())
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(yg, W4.gemm_w4a16(x, p))


def test_fp8_tc_split_pairs_with_busy_sms(cuda):
    """A tcgen05 head whose block pairs are split between CTAs, launched while a long W4 head
    on another stream holds the SMs: its CTAs start in waves, not all at once. The split pairs
    are finished by whichever CTA arrives last, which waits only for CTAs already running, so
    the call completes, with the error word clear and every output identical, bit for bit, to
    the same call made alone."""
    N, K, M = 128 * 301, 2560, 64                  # 151 pairs x 20 K-blocks over 148 SMs: splits
    wq, ws, _ = _fp8_weight(N, K, 21, cuda)
    x = torch.randn(M, K, device=cuda, dtype=torch.bfloat16)
    ref = F8.fp8_lmhead(x, wq, ws)
    torch.cuda.synchronize()
    big = W4.pack_w4a16((torch.randn(151936, K, device=cuda) * 0.02).bfloat16())
    xb = torch.randn(4, K, device=cuda, dtype=torch.bfloat16)
    s_busy, s_head = torch.cuda.Stream(), torch.cuda.Stream()
    for _ in range(3):
        with torch.cuda.stream(s_busy):
            for _ in range(4):
                W4.gemm_w4a16_top(xb, big)
        with torch.cuda.stream(s_head):
            got = F8.fp8_lmhead(x, wq, ws)
        torch.cuda.synchronize()
        for a, b in zip(ref, got):
            assert torch.equal(a, b)
    assert P._lib.lmhead().b200_lmhead_error(1) == 0


@pytest.mark.parametrize("nblk", [296, 297, 298, 301, 447, 1187, 8, 3])
def test_fp8_tc_work_splits(cuda, nblk):
    """Vocabulary sizes around the tcgen05 work split on 148 SMs (whole pairs per CTA, the rest
    split by 128-K units): a pair count that is a multiple of the CTA count (296 blocks = 148
    pairs), one pair more (298 blocks), odd block counts (297, 301), several extra pairs (447,
    1187: the full head) and fewer pairs than SMs (8, 3 blocks: one whole pair per CTA, none
    split). Logits within the reference bound, statistics against the oracle, repeated calls
    identical."""
    N, K, M = 128 * nblk, 2560, 64
    wq, ws, wdq = _fp8_weight(N, K, nblk, cuda)
    g = torch.Generator(device=cuda).manual_seed(10_000 + nblk)       # not the weight's stream
    x = torch.randn(M, K, device=cuda, dtype=torch.bfloat16, generator=g)
    y, mx, arg, lse = F8.fp8_lmhead(x, wq, ws)
    rq, rs = Q.group_quant_fp8(x, 128)
    ref = Q.fp8_block_gemm_ref(rq, rs, wdq)
    rel = ((y.float() - ref).abs().max() / ref.abs().max()).item()
    assert rel < REL_FP8, rel
    _check_stats(f"nblk={nblk}", ref, mx, arg, lse)
    again = F8.fp8_lmhead(x, wq, ws)
    for a, b in zip((y, mx, arg, lse), again):
        assert torch.equal(a, b)
    assert P._lib.lmhead().b200_lmhead_error(1) == 0
    del wdq, ref


@pytest.mark.parametrize("M", [5, 40])
def test_fp8_prepared_step_matches_call(cuda, M):
    """Fp8LmheadStep (buffers checked once, one C call per launch) gives the same logits,
    statistics and packed triples as fp8_lmhead + pack_row_stats, with rotating weights, and
    refuses a weight of another shape."""
    torch.manual_seed(M)
    w1 = (torch.randn(1280, 2560, device=cuda) * 0.02).bfloat16()
    w2 = (torch.randn(1280, 2560, device=cuda) * 0.02).bfloat16()
    packs = [F8.pack_fp8_block(w1), F8.pack_fp8_block(w2)]
    x = torch.randn(M, 2560, device=cuda, dtype=torch.bfloat16)
    out = torch.empty(M, 1280, device=cuda, dtype=torch.bfloat16)
    stats = (torch.empty(M, device=cuda), torch.empty(M, dtype=torch.int64, device=cuda), torch.empty(M, device=cuda))
    packed = torch.empty(M, 3, dtype=torch.float64, device=cuda)
    step = F8.Fp8LmheadStep(x, 1280, vocab_offset=384, out=out, stats_out=stats, packed_out=packed)
    for wq, ws in packs + packs[:1]:
        step(wq, ws)
        y, mx, arg, lse = F8.fp8_lmhead(x, wq, ws, vocab_offset=384)
        torch.cuda.synchronize()
        assert torch.equal(out, y) and torch.equal(stats[0], mx) and torch.equal(stats[1], arg)
        assert torch.equal(stats[2], lse)
        assert torch.equal(packed, P.sharded.pack_row_stats(mx, arg, lse))
    with pytest.raises(ValueError):
        step(packs[0][0][:1152], packs[0][1][:9])
