"""Tensor-core projection GEMM (vmscan_gemm_tf32x3 through the C ABI) against
fp64, with PyTorch's fp32 SIMT GEMM as the fp32 reference (TF32 off): the
same parity rule as every other kernel (tests/parity.py).  Covers the four
operand layouts, ragged tile edges, the K-split path, and the shapes of the
VisionMamba-2D in_proj / out_proj and their gradients."""

import pytest
import torch

from parity import assert_parity

from mlx_vision_mamba_b200 import device_status

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _no_tf32():
    old = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32 = old


def _operand(rows, cols, mn, gen, scale=1.0):
    """A logical (rows x cols) operand stored row-major, or transposed (MN-major)."""
    x = torch.randn(rows, cols, generator=gen, dtype=torch.float64) * scale
    stored = x.t().contiguous() if mn else x.contiguous()
    return x, stored


@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, False), (True, True)])
@pytest.mark.parametrize("m,n,k", [(200, 96, 72), (128, 128, 32), (260, 160, 100), (1568, 512, 384),
                                   # M a multiple of 256 with 128-column tiles: CTA pairs when A is
                                   # MN-major (one item; the second tile's peer half of B partly /
                                   # wholly past N; K split over the pairs)
                                   (256, 128, 64), (512, 200, 100), (768, 132, 4096), (2048, 384, 768)])
def test_gemm_layouts(m, n, k, a_mn, b_mn):
    from mlx_vision_mamba_b200.linear import gemm_tf32x3, tf32_split

    gen = torch.Generator().manual_seed(m * 7 + n * 3 + k + 2 * a_mn + b_mn)
    a, a_st = _operand(m, k, a_mn, gen)
    b, b_st = _operand(n, k, b_mn, gen)
    dev = torch.device("cuda", 0)
    a32 = a_st.float().to(dev)
    b32 = b_st.float().to(dev)
    c = gemm_tf32x3(tf32_split(a32), a_mn, tf32_split(b32), b_mn, m, n, k)
    assert device_status(dev, clear=True) == 0, "a bounded device wait of the GEMM gave up"
    exact = a.float().double() @ b.float().double().t()
    ref32 = (a.float() @ b.float().t())
    assert_parity(f"gemm {m}x{n}x{k} a_mn={a_mn} b_mn={b_mn}", c.cpu(), exact, ref32)


def test_gemm_splitk_out_proj_weight_grad():
    """dW of the 2D model's out_proj: M 384, N 3072, K 12544 (72 tiles, split over K)."""
    from mlx_vision_mamba_b200 import _native
    from mlx_vision_mamba_b200.linear import gemm_tf32x3, tf32_split

    lib = _native.load()
    m, n, k = 384, 3072, 12544
    assert lib.vmscan_gemm_workspace_bytes(m, n, k) > 0
    gen = torch.Generator().manual_seed(5)
    dev = torch.device("cuda", 0)
    dy = torch.randn(k, m, generator=gen).to(dev)
    y = torch.randn(k, n, generator=gen).to(dev)
    c = gemm_tf32x3(tf32_split(dy), True, tf32_split(y), True, m, n, k)
    exact = dy.double().t() @ y.double()
    ref32 = dy.t() @ y
    assert_parity("gemm splitK 384x3072x12544", c, exact, ref32)
    c2 = gemm_tf32x3(tf32_split(dy), True, tf32_split(y), True, m, n, k)
    assert torch.equal(c, c2), "split-K sum is not deterministic"


@pytest.mark.parametrize("t,fin,fout", [(12544, 384, 6144), (12544, 3072, 384), (392, 768, 3072)])
def test_linear_tc_fwd_bwd(t, fin, fout):
    """linear_tc forward, input and weight gradient at the in_proj / out_proj
    shapes of VisionMamba-2D (t = 64 x 196 tokens) and config 1 (2 x 196)."""
    from mlx_vision_mamba_b200.linear import linear_tc

    gen = torch.Generator().manual_seed(t + fin + fout)
    dev = torch.device("cuda", 0)
    x = torch.randn(t, fin, generator=gen).to(dev)
    w = (torch.rand(fout, fin, generator=gen) * 2 - 1).mul_(fin ** -0.5).to(dev)
    dy = torch.randn(t, fout, generator=gen).to(dev)
    xg = x.clone().requires_grad_(True)
    wg = w.clone().requires_grad_(True)
    y = linear_tc(xg, wg)
    y.backward(dy)
    x64, w64, dy64 = x.double(), w.double(), dy.double()
    assert_parity(f"linear_tc y {t}x{fin}->{fout}", y.detach(), x64 @ w64.t(), x @ w.t())
    assert_parity(f"linear_tc dx {t}x{fin}->{fout}", xg.grad, dy64 @ w64, dy @ w)
    assert_parity(f"linear_tc dw {t}x{fin}->{fout}", wg.grad, dy64.t() @ x64, dy.t() @ x)


def test_tf32_split_exact():
    """hi + lo reproduces x to 2^-21 relative, hi and lo carry at most 11 significant bits."""
    from mlx_vision_mamba_b200.linear import tf32_split

    gen = torch.Generator().manual_seed(11)
    x = (torch.randn(1 << 16, generator=gen) * torch.exp(torch.randn(1 << 16, generator=gen) * 4)).cuda()
    hi, lo = tf32_split(x)
    low13 = (1 << 13) - 1
    assert int((hi.view(torch.int32) & low13).abs().sum()) == 0
    assert int((lo.view(torch.int32) & low13).abs().sum()) == 0
    err = (hi.double() + lo.double() - x.double()).abs()
    assert bool((err <= x.double().abs() * 2.0 ** -21).all())


@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (True, True)])
def test_gemm_pair_output_slice_and_accumulate(a_mn, b_mn):
    """M 512 (CTA-pair tiles when A is MN-major) writing a column slice of a
    wider output (ldc 200), then C += A B^T on it; the columns outside the
    slice stay untouched."""
    from mlx_vision_mamba_b200.linear import gemm_tf32x3, tf32_split

    gen = torch.Generator().manual_seed(23 + a_mn)
    dev = torch.device("cuda", 0)
    m, n, k, ld = 512, 160, 96, 200
    a, a_st = _operand(m, k, a_mn, gen)
    b, b_st = _operand(n, k, b_mn, gen)
    a_s, b_s = tf32_split(a_st.float().to(dev)), tf32_split(b_st.float().to(dev))
    out = torch.full((m, ld), 3.0, device=dev)
    gemm_tf32x3(a_s, a_mn, b_s, b_mn, m, n, k, out=out[:, :n])
    exact = a.float().double() @ b.float().double().t()
    assert_parity("pair gemm slice", out[:, :n].cpu(), exact, a.float() @ b.float().t())
    gemm_tf32x3(a_s, a_mn, b_s, b_mn, m, n, k, out=out[:, :n], accumulate=True)
    assert_parity("pair gemm slice accumulate", out[:, :n].cpu(), 2.0 * exact, 2.0 * (a.float() @ b.float().t()))
    assert bool((out[:, n:] == 3.0).all()), "columns outside the output slice were written"
    assert device_status(dev, clear=True) == 0, "a bounded device wait of the GEMM gave up"


def test_gemm_skinny_slices_and_accumulate():
    """The x_proj / dt_proj products of the 2D block (narrow 32- and 64-column
    tiles): operands that are column slices of wider rows, an output slice,
    and C += A B^T."""
    from mlx_vision_mamba_b200.linear import gemm_tf32x3, tf32_split

    gen = torch.Generator().manual_seed(17)
    dev = torch.device("cuda", 0)
    t, dn, r, wide = 12544, 768, 24, 56
    xc = torch.randn(t, dn, generator=gen).to(dev)
    wx = (torch.randn(wide, dn, generator=gen) / dn ** 0.5).to(dev)
    dpre = torch.randn(t, dn, generator=gen).to(dev)
    wdt = (torch.randn(dn, r, generator=gen) / r ** 0.5).to(dev)
    xdbc = torch.randn(t, wide, generator=gen).to(dev)
    du0 = torch.randn(t, dn, generator=gen).to(dev)
    xc_s, xdbc_s, dpre_s = tf32_split(xc), tf32_split(xdbc), tf32_split(dpre)
    # x_proj forward (N 56: 64-column tiles)
    y = gemm_tf32x3(xc_s, False, tf32_split(wx), False, t, wide, dn)
    assert_parity("skinny x_proj fwd", y, xc.double() @ wx.double().t(), xc @ wx.t())
    # dt_proj input gradient into a column slice (N 24: 32-column tiles, ldc 56)
    out = torch.full((t, wide), 7.0, device=dev)
    gemm_tf32x3(dpre_s, False, tf32_split(wdt), True, t, r, dn, out=out[:, :r])
    assert_parity("skinny dt dx", out[:, :r], dpre.double() @ wdt.double(), dpre @ wdt)
    assert bool((out[:, r:] == 7.0).all()), "columns outside the output slice were written"
    # dt_proj weight gradient with B a column slice (row stride 56), K split
    g = gemm_tf32x3(dpre_s, True, (xdbc_s[0][:, :r], xdbc_s[1][:, :r]), True, dn, r, t)
    assert_parity("skinny dt dW", g, dpre.double().t() @ xdbc[:, :r].double(), dpre.t() @ xdbc[:, :r])
    # x_proj input gradient accumulated onto du
    du = du0.clone()
    gemm_tf32x3(xdbc_s, False, tf32_split(wx), True, t, dn, wide, out=du, accumulate=True)
    assert_parity("skinny x_proj dx accumulate", du, du0.double() + xdbc.double() @ wx.double(),
                  du0 + xdbc @ wx)
    # x_proj weight gradient (M 56 < one tile)
    gx = gemm_tf32x3(xdbc_s, True, xc_s, True, wide, dn, t)
    assert_parity("skinny x_proj dW", gx, xdbc.double().t() @ xc.double(), xdbc.t() @ xc)


def test_fused_split_outputs_match_split_pass():
    """The conv forward's xc hi / lo outputs and the dt_proj VJP's dpre hi / lo
    outputs equal vmscan_tf32_split of the fp32 results bit for bit, and the
    dbias partials do not change."""
    import ctypes

    from mlx_vision_mamba_b200 import _native, directions_for
    from mlx_vision_mamba_b200.linear import tf32_split

    lib = _native.load()
    dev = torch.device("cuda", 0)
    gen = torch.Generator().manual_seed(23)
    b, l, c, k = 3, 196, 128, 4
    x = torch.randn(b, l, c, generator=gen).to(dev)
    w = torch.randn(c, k, 1, generator=gen).to(dev)
    bias = torch.randn(c, generator=gen).to(dev)
    S = _native.Strides(l * c, c)
    sp = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    direction = directions_for(4, (14, 14))[2]
    dref = ctypes.byref(direction.to_native())
    out, hi, lo = (torch.empty_like(x) for _ in range(3))
    assert lib.vmscan_conv1d_silu_fwd(b, l, c, k, P(x), S, P(w), P(bias), P(out), S, P(hi), P(lo), dref, sp) == 0
    out2 = torch.empty_like(x)
    assert lib.vmscan_conv1d_silu_fwd(b, l, c, k, P(x), S, P(w), P(bias), P(out2), S, None, None, dref, sp) == 0
    h_ref, l_ref = tf32_split(out2)
    assert torch.equal(out, out2) and torch.equal(hi, h_ref) and torch.equal(lo, l_ref)

    ntok, r, dn, wide = 300, 24, 256, 56
    xw = torch.randn(ntok, wide, generator=gen).to(dev)
    wdt = (torch.randn(dn, r, generator=gen) / r ** 0.5).to(dev)
    bdt = torch.randn(dn, generator=gen).to(dev)
    gin = torch.randn(ntok, dn, generator=gen).to(dev)
    rows = lib.vmscan_dt_softplus_bias_rows(ntok)
    dpre, part = torch.empty(ntok, dn, device=dev), torch.empty(rows, dn, device=dev)
    dhi, dlo, part2 = torch.empty(ntok, dn, device=dev), torch.empty(ntok, dn, device=dev), torch.empty(rows, dn,
                                                                                                        device=dev)
    assert lib.vmscan_dt_softplus_bwd(ntok, r, dn, P(xw), wide, P(wdt), P(bdt), P(gin), dn, P(dpre), dn, None,
                                      P(part), sp) == 0
    assert lib.vmscan_dt_softplus_bwd(ntok, r, dn, P(xw), wide, P(wdt), P(bdt), P(gin), dn, P(dhi), dn, P(dlo),
                                      P(part2), sp) == 0
    h_ref, l_ref = tf32_split(dpre)
    assert torch.equal(dhi, h_ref) and torch.equal(dlo, l_ref) and torch.equal(part, part2)


def test_scan_and_conv_vjp_split_outputs_match_split_pass():
    """y_lo of vmscan_fwd, dz_lo of vmscan_bwd and dx_lo of
    vmscan_conv1d_silu_bwd: hi written over the fp32 output and lo beside it
    equal vmscan_tf32_split of the plain outputs bit for bit, with every other
    output unchanged (a direction with chunking over L and a permuted order)."""
    import ctypes

    from mlx_vision_mamba_b200 import _native, directions_for
    from mlx_vision_mamba_b200.linear import tf32_split

    lib = _native.load()
    dev = torch.device("cuda", 0)
    gen = torch.Generator().manual_seed(29)
    b, l, dn = 2, 196, 256
    sp = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    P = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else None  # noqa: E731
    S = lambda t: _native.Strides(t.stride(0), t.stride(1))  # noqa: E731
    t = {"u": torch.randn(b, l, dn, generator=gen), "z": torch.randn(b, l, dn, generator=gen),
         "delta": torch.nn.functional.softplus(torch.randn(b, l, dn, generator=gen) * 0.5 - 3),
         "A": -torch.rand(dn, 16, generator=gen) * 4, "B": torch.randn(b, l, 16, generator=gen),
         "C": torch.randn(b, l, 16, generator=gen), "D": torch.randn(dn, generator=gen),
         "dy": torch.randn(b, l, dn, generator=gen)}
    t = {k: v.to(dev).contiguous() for k, v in t.items()}
    dref = ctypes.byref(directions_for(4, (14, 14))[3].to_native())
    n_ck = lib.vmscan_ckpt_elems(b, l, dn, 16, dref)
    fws_n = lib.vmscan_fwd_workspace_bytes(b, l, dn, 16, dref)
    fws = torch.empty(max(fws_n, 16), dtype=torch.uint8, device=dev)

    def fwd(split):
        y, ylo, ck = torch.empty_like(t["u"]), (torch.empty_like(t["u"]) if split else None), torch.empty(n_ck, device=dev)
        assert lib.vmscan_fwd(b, l, dn, 16, P(t["u"]), S(t["u"]), P(t["delta"]), S(t["delta"]), P(t["A"]), P(t["B"]),
                              S(t["B"]), P(t["C"]), S(t["C"]), P(t["D"]), P(t["z"]), S(t["z"]), P(y), S(y), P(ylo),
                              P(ck), dref, P(fws), fws_n, sp) == 0
        return y, ylo, ck

    y, _, ck = fwd(False)
    yhi, ylo, ck2 = fwd(True)
    h_ref, l_ref = tf32_split(y)
    assert torch.equal(yhi, h_ref) and torch.equal(ylo, l_ref) and torch.equal(ck, ck2)

    ws_n = lib.vmscan_bwd_workspace_bytes(b, l, dn, 16, dref, 0)
    ws = torch.empty(ws_n, dtype=torch.uint8, device=dev)

    def bwd(split):
        o = {k: torch.empty_like(t["u"]) for k in ("du", "ddelta", "dz")}
        o["dzlo"] = torch.empty_like(t["u"]) if split else None
        o["dA"], o["dD"] = torch.empty(dn, 16, device=dev), torch.empty(dn, device=dev)
        o["dB"], o["dC"] = torch.empty(b, l, 16, device=dev), torch.empty(b, l, 16, device=dev)
        assert lib.vmscan_bwd(b, l, dn, 16, P(t["u"]), S(t["u"]), P(t["delta"]), S(t["delta"]), P(t["A"]), P(t["B"]),
                              S(t["B"]), P(t["C"]), S(t["C"]), P(t["D"]), P(t["z"]), S(t["z"]), P(ck), P(t["dy"]),
                              S(t["dy"]), P(o["du"]), S(o["du"]), P(o["ddelta"]), S(o["ddelta"]), P(o["dA"]),
                              P(o["dB"]), S(o["dB"]), P(o["dC"]), S(o["dC"]), P(o["dD"]), P(o["dz"]), S(o["dz"]),
                              P(o["dzlo"]), dref, P(ws), ws_n, sp) == 0
        return o

    a, s_ = bwd(False), bwd(True)
    h_ref, l_ref = tf32_split(a["dz"])
    assert torch.equal(s_["dz"], h_ref) and torch.equal(s_["dzlo"], l_ref)
    for k in ("du", "ddelta", "dA", "dB", "dC", "dD"):
        assert torch.equal(a[k], s_[k]), k

    k = 4
    w = torch.randn(dn, k, 1, generator=gen).to(dev)
    bias = torch.randn(dn, generator=gen).to(dev)
    cws_n = lib.vmscan_conv1d_bwd_workspace_bytes(b, l, dn, k)
    cws = torch.empty(cws_n, dtype=torch.uint8, device=dev)

    def cbwd(split):
        dx, dxlo = torch.empty_like(t["u"]), (torch.empty_like(t["u"]) if split else None)
        dw, db = torch.empty_like(w), torch.empty_like(bias)
        assert lib.vmscan_conv1d_silu_bwd(b, l, dn, k, P(t["u"]), S(t["u"]), P(w), P(bias), P(t["dy"]), S(t["dy"]),
                                          P(dx), S(dx), P(dxlo), P(dw), P(db), dref, P(cws), cws_n, sp) == 0
        return dx, dxlo, dw, db

    dx, _, dw, db = cbwd(False)
    dxhi, dxlo, dw2, db2 = cbwd(True)
    h_ref, l_ref = tf32_split(dx)
    assert torch.equal(dxhi, h_ref) and torch.equal(dxlo, l_ref) and torch.equal(dw, dw2) and torch.equal(db, db2)


def test_tf32_split_many_matches_split():
    """vmscan_tf32_split_multi (one launch, several tensors) equals
    vmscan_tf32_split per tensor bit for bit."""
    from mlx_vision_mamba_b200.linear import tf32_split, tf32_split_many

    gen = torch.Generator().manual_seed(31)
    xs = [torch.randn(n, generator=gen).cuda() for n in (4, 56 * 768, 384 * 6144, 768 * 24, 1000)]
    many = tf32_split_many(xs)
    for x, (h, l) in zip(xs, many):
        h_ref, l_ref = tf32_split(x)
        assert torch.equal(h, h_ref) and torch.equal(l, l_ref)
    xs20 = [torch.randn(8 * (i + 1), generator=gen).cuda() for i in range(20)]  # more than one launch's 16
    for x, (h, l) in zip(xs20, tf32_split_many(xs20)):
        assert torch.equal(h, tf32_split(x)[0]) and torch.equal(l, tf32_split(x)[1])
