"""Pedazen on the GPU: every kernel of the design against its plain twin, and the whole engine (step function,
cache manager, captured steps, scheduler and entry point) against the plain implementation, in both precisions."""

from types import SimpleNamespace

import pytest
import torch

import helpers
import pedazen_cases as cases
import plain_pedazen
from test_pedazen import check_one_key_carries_the_weight
from torch_kernels import TorchKernels
from tt_transformers_b200.config import EngineConfig
from tt_transformers_b200.engine.step import StepEntry, build_engine
from tt_transformers_b200.parts import PagedKV
from tt_transformers_b200.parts.base import RecurrentState, SlotState

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
TOL = {torch.float32: 2e-5, torch.bfloat16: 2e-2}


@pytest.fixture(scope="module")
def kernels():
    from tt_transformers_b200.kernels import load_kernels
    return load_kernels(torch.device(DEV))


@pytest.fixture(scope="module")
def twin():
    return TorchKernels(DEV)


def _close(got, ref, tol):
    assert got.shape == ref.shape
    assert not torch.isnan(got.float()).any()
    err = float((got.float() - ref.float()).abs().max()) / max(float(ref.float().abs().max()), 1e-6)
    assert err < tol, err


def _batch(segs, slots=None):
    """segs: [(cached tokens, new tokens)] -> what the kernels read of a StepBatch."""
    lens, pos0 = [n for _, n in segs], [p for p, _ in segs]
    slots = slots if slots is not None else list(range(len(segs)))
    cu = [0]
    for n in lens:
        cu.append(cu[-1] + n)
    i32 = dict(dtype=torch.int32, device=DEV)
    return SimpleNamespace(
        positions=torch.cat([torch.arange(p, p + n) for p, n in segs]).to(**i32),
        seg_of_token=torch.cat([torch.full((n,), r) for r, n in enumerate(lens)]).to(**i32),
        cu_seqlens=torch.tensor(cu, **i32), seg_pos0=torch.tensor(pos0, **i32), seg_slot=torch.tensor(slots, **i32),
        seg_lens=lens, seg_pos0_list=pos0, seg_slot_list=slots, num_segments=len(segs), num_tokens=cu[-1],
        max_seg_len=max(lens), max_context=max(p + n for p, n in segs), extras={})


# ---------------------------------------------------------------------------- the stream and the norms
@pytest.mark.parametrize("width", [60, 128, 1000, 4096])
def test_stream_add_norm(kernels, twin, width):
    g = torch.Generator().manual_seed(width)
    for deltas, vec, weight, offset in (([torch.float32, torch.bfloat16], False, True, 1.0), ([torch.bfloat16], True, True, 0.0),
                                        ([], True, False, 0.0), ([torch.float32] * 3, False, True, 1.0), ([], False, True, 1.0)):
        x = (2 * torch.randn(5, width, generator=g)).to(DEV)
        ds = [torch.randn(5, width, generator=g).to(DEV, dt) for dt in deltas]
        v = torch.randn(width, generator=g).to(DEV) if vec else None
        w = (0.3 * torch.randn(width, generator=g)).to(DEV) if weight else None
        for out_dtype in (torch.float32, torch.bfloat16):
            x_ref, x_got = x.clone(), x.clone()
            ref = twin.stream_add_norm(x_ref, ds, row_vector=v, weight=w, eps=1e-5, offset=offset, out_dtype=out_dtype)
            got = kernels.stream_add_norm(x_got, ds, row_vector=v, weight=w, eps=1e-5, offset=offset, out_dtype=out_dtype)
            _close(x_got, x_ref, 1e-6)
            if weight:
                _close(got, ref, TOL[out_dtype])
            else:
                assert got is None


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("width", [36, 512, 3000])
def test_gated_norm_pair_norm_and_activations(kernels, twin, dtype, width):
    g = torch.Generator().manual_seed(width)
    x = torch.randn(7, width, generator=g).to(DEV) * 3
    wide = torch.randn(7, 2 * width + 8, generator=g).to(DEV, dtype)
    w = (1 + 0.3 * torch.randn(width, generator=g)).to(DEV)
    gate = wide[:, width + 8:]                                     # a slice of a wider product
    _close(kernels.gated_rmsnorm(x, w, 1e-5, gate, dtype), twin.gated_rmsnorm(x, w, 1e-5, gate, dtype), TOL[dtype])
    a, b = torch.randn(7, width, generator=g).to(DEV, dtype), (5 * torch.randn(7, width, generator=g)).to(DEV, dtype)
    w2 = (1 + 0.3 * torch.randn(width, generator=g)).to(DEV)
    _close(kernels.mean_rmsnorm_pair(a, w, b, w2, 1e-5), twin.mean_rmsnorm_pair(a, w, b, w2, 1e-5), 2e-5)
    gu = (2 * torch.randn(7, 2 * width, generator=g)).to(DEV, dtype)
    for act in ("silu", "gelu_tanh"):
        _close(kernels.glu_activation(gu, act), twin.glu_activation(gu, act), TOL[dtype])
    pre = (2 * torch.randn(7, width, generator=g)).to(DEV)
    _close(kernels.activation(pre, "relu2", dtype), twin.activation(pre, "relu2", dtype), TOL[dtype])


# ---------------------------------------------------------------------------- lightning attention
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("H,D,V", [(3, 32, 48), (1, 10, 6), (3, 48, 20), (2, 128, 64), (5, 72, 136), (2, 256, 8)])
def test_lightning_attention_against_its_twin(kernels, twin, dtype, H, D, V):
    """Portions beside single tokens, continuing from a state that is not zero, on slots in any order; a second step
    continues from what the first left; a state that must only be read stays as it was."""
    g = torch.Generator().manual_seed(H * D + V)
    segs = [(0, 37), (90, 1), (5, 2), (0, 1), (300, 70), (0, 200)]
    slots = [3, 0, 5, 1, 4, 6]
    decays = torch.tensor([1.0, 0.0, 0.999, 0.6, 0.9][:H] if H <= 5 else [0.9] * H, device=DEV)
    state = (torch.randn(8, H, D, V, generator=g) * 0.5).to(DEV)
    for step in range(2):
        batch = _batch(segs, slots)
        proj = torch.randn(batch.num_tokens, 2 * H * D + 2 * H * V + 3, generator=g).to(DEV, dtype)
        s_ref, s_got = state.clone(), state.clone()
        v_ref = SlotState((H, D, V)).view({"state": s_ref}, slots=batch.seg_slot, slot_list=slots)
        v_got = SlotState((H, D, V)).view({"state": s_got}, slots=batch.seg_slot, slot_list=slots)
        ref = twin.lightning_attention(proj, batch, v_ref, H, D, V, decays)
        got = kernels.lightning_attention(proj, batch, v_got, H, D, V, decays)
        # float32 arithmetic on the same inputs; the chunked form rounds the activations to bfloat16 first
        _close(got, ref, 5e-5 if dtype == torch.float32 else 1e-2)
        _close(s_got, s_ref, 5e-5 if dtype == torch.float32 else 1e-2)
        assert torch.equal(s_got[[2, 7]], state[[2, 7]])                   # nobody's slots are nobody's
        kept = s_got.clone()
        kernels.lightning_attention(proj, batch, v_got, H, D, V, decays, write_state=False)
        assert torch.equal(s_got, kept)
        state = s_got


@pytest.mark.parametrize("H,D,V", [(2, 128, 64), (3, 48, 20), (1, 16, 40), (2, 256, 32)])
def test_lightning_chunks_keep_float32_where_the_recurrence_does(kernels, H, D, V):
    """Pre-activations from 20 on are their own silu in float32 and exact in bfloat16, so nothing but the arithmetic
    differs between the chunked form and the walk token by token: decays, state and weights must agree to float32
    rounding and the two-halves splitting (2^-17), not to bfloat16's."""
    g = torch.Generator().manual_seed(D + V)
    segs, slots = [(0, 150), (40, 17), (3, 64), (9, 65)], [2, 0, 1, 3]
    decays = torch.tensor([0.999, 0.9, 0.6][:H], device=DEV)
    batch = _batch(segs, slots)
    proj = torch.randint(20, 29, (batch.num_tokens, 2 * H * D + 2 * H * V), generator=g).to(DEV, torch.bfloat16)
    state = (torch.randn(4, H, D, V, generator=g) * 1e4).to(DEV)
    results = []
    for chunks in (True, False):
        kernels.use_lightning_chunks = chunks
        try:
            s_now = state.clone()
            view = SlotState((H, D, V)).view({"state": s_now}, slots=batch.seg_slot, slot_list=slots)
            results.append((kernels.lightning_attention(proj, batch, view, H, D, V, decays), s_now))
        finally:
            kernels.use_lightning_chunks = True
    _close(results[0][0], results[1][0], 3e-5)
    _close(results[0][1], results[1][1], 3e-5)


# ---------------------------------------------------------------------------- the recurrent block
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("C,B,taps", [(192, 6, 4), (30, 1, 1), (20, 5, 6), (96, 3, 2), (520, 2, 9)])
def test_convolution_and_recurrence_against_their_twins(kernels, twin, dtype, C, B, taps):
    """Portions shorter and longer than the convolution's reach, single tokens, first tokens; two steps in a row."""
    g = torch.Generator().manual_seed(C + taps)
    segs = [(0, 23), (40, 1), (7, 2), (0, 1), (11, 3), (64, 50), (9, 300)]
    slots = [2, 0, 5, 1, 6, 3, 7]
    s = C // B
    req = RecurrentState(C, taps)
    state = torch.randn(9, C, generator=g).to(DEV)
    tail = torch.randn(9, max(taps - 1, 1), C, generator=g).to(DEV, dtype)
    conv_w, conv_b = (torch.randn(C, taps, generator=g) * 0.5).to(DEV), (torch.randn(C, generator=g) * 0.3).to(DEV)
    b_in = (torch.randn(2 * C, generator=g) * 0.3).to(DEV)
    w_gates = (torch.randn(B, 2 * s, s, generator=g) * s ** -0.5).to(DEV, dtype)
    b_gates, rate = (torch.randn(B, 2 * s, generator=g) * 0.3).to(DEV), (8 * torch.rand(C, generator=g)).to(DEV)
    for step in range(2):
        batch = _batch(segs, slots)
        yx = torch.randn(batch.num_tokens, 2 * C, generator=g).to(DEV, dtype)
        st_ref, st_got, tl_ref, tl_got = state.clone(), state.clone(), tail.clone(), tail.clone()
        v_ref = req.view({"state": st_ref, "tail": tl_ref}, slots=batch.seg_slot, slot_list=slots)
        v_got = req.view({"state": st_got, "tail": tl_got}, slots=batch.seg_slot, slot_list=slots)
        u_ref = twin.causal_conv(yx[:, C:], b_in[C:], conv_w, conv_b, batch, v_ref)
        u_got = kernels.causal_conv(yx[:, C:], b_in[C:], conv_w, conv_b, batch, v_got)
        _close(u_got, u_ref, TOL[dtype])
        g_ref = twin.heads_linear(u_ref.view(-1, B, s), w_gates, out_dtype=torch.float32)
        g_got = kernels.heads_linear(u_ref.view(-1, B, s), w_gates, out_dtype=torch.float32)
        assert g_got.dtype == torch.float32
        _close(g_got, g_ref, 2e-5)                       # float32 sums also of a bfloat16 product
        ref = twin.gated_recurrence(u_ref, g_ref, b_gates, rate, yx, b_in, batch, v_ref)
        got = kernels.gated_recurrence(u_ref, g_got, b_gates, rate, yx, b_in, batch, v_got)
        _close(got, ref, TOL[dtype])
        _close(st_got, st_ref, 2e-5)
        if taps > 1:
            _close(tl_got, tl_ref, 1e-6)
        assert torch.equal(st_got[[4, 8]], state[[4, 8]])
        state, tail = st_got, tl_got


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("C,B,taps", [(192, 6, 4), (30, 1, 1), (20, 5, 6), (96, 3, 2), (1040, 2, 9)])
def test_a_decoded_token_in_one_kernel_against_the_three(kernels, twin, dtype, C, B, taps):
    """Single tokens at a request's start and later, on slots in any order, three steps in a row."""
    g = torch.Generator().manual_seed(C + taps)
    segs, slots = [(0, 1), (40, 1), (7, 1), (300, 1)], [2, 0, 5, 3]
    s = C // B
    req = RecurrentState(C, taps)
    state = torch.randn(7, C, generator=g).to(DEV)
    tail = torch.randn(7, max(taps - 1, 1), C, generator=g).to(DEV, dtype)
    conv_w, conv_b = (torch.randn(C, taps, generator=g) * 0.5).to(DEV), (torch.randn(C, generator=g) * 0.3).to(DEV)
    b_in = (torch.randn(2 * C, generator=g) * 0.3).to(DEV)
    w_gates = (torch.randn(B, 2 * s, s, generator=g) * s ** -0.5).to(DEV, dtype)
    b_gates, rate = (torch.randn(B, 2 * s, generator=g) * 0.3).to(DEV), (8 * torch.rand(C, generator=g)).to(DEV)
    st_ref, st_got, tl_ref, tl_got = state.clone(), state.clone(), tail.clone(), tail.clone()
    for step in range(3):
        batch = _batch(segs, slots)
        yx = torch.randn(batch.num_tokens, 2 * C, generator=g).to(DEV, dtype)
        v_ref = req.view({"state": st_ref, "tail": tl_ref}, slots=batch.seg_slot, slot_list=slots)
        v_got = req.view({"state": st_got, "tail": tl_got}, slots=batch.seg_slot, slot_list=slots)
        ref = twin.recurrent_token(yx, b_in, conv_w, conv_b, w_gates, b_gates, rate, batch, v_ref)
        got = kernels.recurrent_token(yx, b_in, conv_w, conv_b, w_gates, b_gates, rate, batch, v_got)
        _close(got, ref, TOL[dtype])
        _close(st_got, st_ref, 2e-5 if dtype == torch.float32 else 2e-2)
        if taps > 1:
            _close(tl_got, tl_ref, 1e-6)
        assert torch.equal(st_got[[1, 4, 6]], state[[1, 4, 6]])
        kept_state, kept_tail = st_got.clone(), tl_got.clone()
        kernels.recurrent_token(yx, b_in, conv_w, conv_b, w_gates, b_gates, rate, batch, v_got, write_state=False)
        assert torch.equal(st_got, kept_state) and torch.equal(tl_got, kept_tail)


# ---------------------------------------------------------------------------- attention with a sink, a cap and chunks
def _attention_setup(segs, heads, kv_heads, dim, vdim, page, chunk, window, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    width = max(-(-(p + n) // page) for p, n in segs)
    total = sum(-(-(p + n) // page) for p, n in segs)
    order = (torch.randperm(total, generator=g) + 1).tolist()
    keys = torch.full((total + 1, kv_heads, page, dim), float("nan"))
    values = torch.full((total + 1, kv_heads, page, vdim), float("nan"))
    table = torch.zeros(len(segs), width, dtype=torch.int32)
    at = 0
    for r, (p, n) in enumerate(segs):
        for i in range(-(-(p + n) // page)):
            table[r, i] = order[at]
            fill = min(page, p - i * page)                  # the cached tokens only: the new ones are written by the kernel
            if fill > 0:
                keys[order[at], :, :fill] = torch.randn(kv_heads, fill, dim, generator=g)
                values[order[at], :, :fill] = torch.randn(kv_heads, fill, vdim, generator=g)
            at += 1
    view = PagedKV(kv_heads, dim, window, value_dim=vdim, chunk=chunk).view(
        {"keys": keys.to(DEV, dtype), "values": values.to(DEV, dtype)}, block_table=table.to(DEV), page_size=page)
    batch = _batch(segs)
    qkv = torch.randn(batch.num_tokens, (heads + kv_heads) * dim + kv_heads * vdim, generator=g).to(DEV, dtype)
    return batch, view, qkv, g


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("heads,kv_heads,dim,vdim,rot,page,chunk,window", [
    (6, 6, 80, 80, 40, 16, 112, None), (4, 2, 32, 16, 16, 4, 24, None), (1, 1, 10, 7, 6, 8, 7, None), (5, 5, 6, 9, 2, 16, 1, None),
    (6, 1, 16, 48, 16, 16, 16, None), (3, 1, 64, 128, 0, 32, None, None), (2, 2, 24, 40, 24, 16, 50, 20), (4, 4, 136, 264, 8, 16, None, 33),
    (8, 2, 64, 64, 32, 16, 96, None), (4, 1, 128, 128, 128, 16, None, 100), (6, 3, 64, 64, 0, 32, 200, None), (2, 2, 128, 128, 64, 8, 33, None)])
def test_sink_attention_against_its_twin(kernels, twin, dtype, heads, kv_heads, dim, vdim, rot, page, chunk, window):
    segs = [(0, 70), (129, 1), (63, 2), (64, 1), (0, 1), (300, 1), (127, 3), (page - 1, 2), (15, 40), (95, 3), (96, 1)]
    batch, view, qkv, g = _attention_setup(segs, heads, kv_heads, dim, vdim, page, chunk, window, dtype, seed=heads * dim + vdim)
    ref_view = PagedKV(kv_heads, dim, window, value_dim=vdim, chunk=chunk).view(
        {"keys": view.keys.clone(), "values": view.values.clone()}, block_table=view.block_table, page_size=page)
    q_w, k_w = (1 + 0.3 * torch.randn(dim, generator=g)).to(DEV), (1 + 0.3 * torch.randn(dim, generator=g)).to(DEV)
    inv_freq = (1.0 / 1000.0 ** (torch.arange(0, rot, 2).float() / rot)).to(DEV) if rot else None
    sinks = (torch.randn(heads, generator=g) * 2).to(DEV)
    for norms in ((q_w, k_w), (None, None)):
        a, b = qkv.clone(), qkv.clone()
        twin.qk_norm_rope_write(a, batch, norms[0], norms[1], 1e-5, inv_freq, rot, heads, kv_heads, dim, vdim, ref_view)
        kernels.qk_norm_rope_write(b, batch, norms[0], norms[1], 1e-5, inv_freq, rot, heads, kv_heads, dim, vdim, view)
        _close(b[:, :(heads + kv_heads) * dim], a[:, :(heads + kv_heads) * dim], TOL[dtype])
        written = ~torch.isnan(ref_view.keys.float())
        assert torch.equal(written, ~torch.isnan(view.keys.float()))
        _close(torch.where(written, view.keys.float(), 0), torch.where(written, ref_view.keys.float(), 0), TOL[dtype])
        wv = ~torch.isnan(ref_view.values.float())
        assert torch.equal(torch.where(wv, view.values.float(), 0), torch.where(wv, ref_view.values.float(), 0))
        for cap, use_sinks in ((20.0, sinks), (None, sinks), (3.0, None)):
            ref = twin.sink_attention(a, batch, heads, kv_heads, dim, vdim, 0.3, cap, use_sinks, ref_view)
            got = kernels.sink_attention(a, batch, heads, kv_heads, dim, vdim, 0.3, cap, use_sinks, ref_view)
            _close(got, ref, TOL[dtype])
    more = kernels.sink_attention(a, batch, heads, kv_heads, dim, vdim, 0.3, 3.0, sinks + 3.0, ref_view)
    assert float((more.float() - got.float()).abs().max()) > 0.02          # a sink that is left out shows


@pytest.mark.parametrize("heads,kv_heads,dim,page,chunk", [(8, 2, 64, 16, None), (4, 1, 128, 16, 600), (6, 3, 64, 32, 256), (2, 2, 128, 16, 1024)])
def test_sink_attention_over_long_contexts_with_key_splits(kernels, twin, heads, kv_heads, dim, page, chunk):
    """Contexts long enough for the tensor-core kernel to cut a query's keys into splits that are merged afterwards:
    the sink joins the denominator once, whichever split holds it; decoded tokens and prompt portions."""
    for segs in ([(1100, 1), (700, 1)], [(0, 700)], [(600, 3), (511, 2), (1023, 1), (1024, 1)]):
        batch, view, qkv, g = _attention_setup(segs, heads, kv_heads, dim, dim, page, chunk, None, torch.bfloat16, seed=dim + len(segs))
        sinks = (torch.randn(heads, generator=g) * 2 + 2).to(DEV)
        twin.qk_norm_rope_write(qkv, batch, None, None, 1e-5, None, 0, heads, kv_heads, dim, dim, view)
        for cap, use_sinks in ((25.0, sinks), (None, None)):
            ref = twin.sink_attention(qkv, batch, heads, kv_heads, dim, dim, 0.2, cap, use_sinks, view)
            got = kernels.sink_attention(qkv, batch, heads, kv_heads, dim, dim, 0.2, cap, use_sinks, view)
            _close(got, ref, 2e-2)
            kernels.use_mma_attention = False                   # the float32-arithmetic kernel on the same pages
            try:
                _close(kernels.sink_attention(qkv, batch, heads, kv_heads, dim, dim, 0.2, cap, use_sinks, view), ref, 2e-2)
            finally:
                kernels.use_mma_attention = True


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_one_key_carries_the_weight_inside_its_chunk_only(kernels, dtype):
    check_one_key_carries_the_weight(kernels, DEV, dtype)


# ---------------------------------------------------------------------------- the router and the experts
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("width,E,top,groups,keep,inter,T", [(192, 10, 3, 5, 3, 80, 70), (60, 1, 1, 1, 1, 20, 5), (128, 9, 1, 3, 3, 9, 33),
                                                           (64, 8, 2, 4, 2, 48, 300), (512, 32, 8, 8, 4, 128, 1100), (48, 6, 3, 2, 1, 40, 3)])
def test_grouped_router_and_plain_experts_against_their_twins(kernels, twin, dtype, width, E, top, groups, keep, inter, T):
    g = torch.Generator().manual_seed(width + E)
    x = torch.randn(T, width, generator=g).to(DEV, dtype)
    w_r = (torch.randn(E, width, generator=g) * 4 * width ** -0.5).to(DEV)
    c_ref, w_ref = twin.route_grouped(x, w_r, E, top, groups, keep, 1e-20)
    c_got, w_got = kernels.route_grouped(x, w_r, E, top, groups, keep, 1e-20)
    assert torch.equal(c_got, c_ref)
    _close(w_got, w_ref, 1e-5)
    assert float((w_got.sum(-1) - 1).abs().max()) < 1e-5
    # every choice lies in one of the `keep` best groups
    scores = torch.softmax(x.float() @ w_r.t(), -1)
    best = scores.view(T, groups, E // groups).max(-1).values
    kept = best.topk(keep, -1).indices
    assert bool((kept[:, None, :] == (c_got.long() // (E // groups))[:, :, None]).any(-1).all())
    w_up = (torch.randn(E, inter, width, generator=g) * width ** -0.5).to(DEV, dtype)
    w_down = (torch.randn(E, width, inter, generator=g) * inter ** -0.5).to(DEV, dtype)
    rows = min(T, 64)            # the twin walks pair by pair
    ref = twin.plain_experts(x[:rows], c_ref[:rows], w_ref[:rows], w_up, w_down)
    got = kernels.plain_experts(x, c_got, w_got, w_up, w_down)
    _close(got[:rows], ref, TOL[dtype])
    few = kernels.plain_experts(x[:5], c_got[:5], w_got[:5], w_up, w_down)          # the matrix-vector form
    _close(few, ref[:5], TOL[dtype])


# ---------------------------------------------------------------------------- the whole engine
def _plain(cfg, w, toks):
    return plain_pedazen.forward(cfg, w, toks).float()


@pytest.mark.parametrize("dtype,tol", [("float32", 1e-4), ("bfloat16", 6e-2)])
@pytest.mark.parametrize("name", ["ALIGNED", "ODD", "PLAIN", "TENSOR"])
def test_engine_matches_the_plain_implementation(tmp_path, dtype, tol, name):
    folder = cases.write_folder(str(tmp_path / name), getattr(cases, name), seed=3,
                                dtype=torch.float32 if dtype == "float32" else torch.bfloat16)
    cfg, w = cases.read_folder(folder)
    requests = {f"r{i}": helpers.random_tokens(cfg["vocab"], n, 70 + i) for i, n in enumerate((37, 1, 19, 8, 26, 2, 140))}
    ref = {rid: _plain(cfg, w, toks) for rid, toks in requests.items()}
    for make_steps in (helpers.steps_whole, helpers.steps_decode_tail, helpers.steps_portions, helpers.steps_mixed):
        for graphs in (True, False):
            steps = make_steps(requests)
            pages = -(-helpers.max_live_tokens(requests, steps, rounding=16) // 16)
            engine = build_engine(folder, EngineConfig(dtype=dtype, page_size=16, num_pages=pages, max_batch_size=4,
                                                       max_seq_len=256, cuda_graph=graphs, device=DEV))
            for grp in engine.cache.groups:
                for t in grp.storage.values():
                    t.fill_(float("nan"))
            got = helpers.run_steps(engine, steps)
            engine.cache.audit()
            assert engine.cache.free_pages() == pages and engine.cache.free_slots == 4
            for rid in ref:
                if dtype == "float32":
                    assert helpers.relative_error(got[rid], ref[rid]) < tol, (make_steps.__name__, graphs, rid)
                else:
                    # in bfloat16 a router's close call may go the other way for a token or two: nine rows in ten
                    # must agree, and the typical row closely
                    scale = float(ref[rid].abs().max())
                    rows = (got[rid] - ref[rid]).abs().amax(dim=-1) / scale
                    assert float((rows < tol).float().mean()) >= 0.9 and float(rows.median()) < tol / 2, (make_steps.__name__, graphs, rid)
            engine.close()


def test_long_decoding_through_captured_steps(tmp_path):
    """300 decoded tokens after a prompt of 40, three requests side by side: state, convolution tails, chunk edges and
    the pages given back behind them, step after step through replays of captured steps."""
    folder = cases.write_folder(str(tmp_path / "m"), cases.ALIGNED, seed=9)
    cfg, w = cases.read_folder(folder)
    requests = {f"r{i}": helpers.random_tokens(cfg["vocab"], 340 - 7 * i, 20 + i) for i in range(3)}
    ref = {rid: _plain(cfg, w, toks) for rid, toks in requests.items()}
    steps = helpers.steps_many(requests, live=3, tail=300, portion=(2, 40))
    engine = build_engine(folder, EngineConfig(dtype="float32", page_size=16, num_pages=3 * 5, max_batch_size=4, max_seq_len=512,
                                               device=DEV))
    got = helpers.run_steps(engine, steps)
    assert engine.graphs is not None and engine.graphs.replays >= 290
    places = helpers.wanted_positions(steps)
    for rid in ref:
        assert helpers.relative_error(got[rid], ref[rid][places[rid]]) < 2e-4, rid
    engine.cache.audit()


def test_greedy_generation_through_the_entry_point(tmp_path):
    from tt_transformers_b200.engine.llm import from_pretrained

    folder = cases.write_folder(str(tmp_path / "g"), cases.PLAIN, seed=7)
    cfg, w = cases.read_folder(folder)
    prompts = [helpers.random_tokens(cfg["vocab"], n, 80 + n) for n in (4, 13, 21, 50)]

    def plain_greedy(prompt, new):
        toks = list(prompt)
        for _ in range(new):
            toks.append(int(_plain(cfg, w, toks)[-1].argmax()))
        return toks[len(prompt):]

    expect = [plain_greedy(p, 12) for p in prompts]
    # pages of 8 tokens, not enough for all four requests at their full length: one gives way and is recomputed
    llm = from_pretrained(folder, dtype="float32", page_size=8, num_pages=16, max_batch_size=4, max_seq_len=128,
                          max_step_tokens=32, max_chunk_tokens=16, device=DEV)
    assert llm.generate(prompts, max_new_tokens=12) == expect
    llm.engine.cache.audit()
    assert llm.engine.cache.free_pages() == 16
