"""The TMA-staged forward (long token streams) against the register-staged
forward and the oracle: both implementations run the same arithmetic, so
their outputs must be bit-identical; the kernels must record no device error
(a pipeline wait that timed out)."""
import numpy as np
import pytest
import torch

from gpu_helpers import DEV, assert_close, rand, ragged_cu, to_np
from oracle import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture
def capi():
    from greta_plugin_b200 import _capi

    _capi.device_errors(clear=True)
    yield _capi
    assert _capi.device_errors(clear=True) == 0


def both(capi, fn):
    a = fn()
    torch.cuda.synchronize()
    with capi.launch_options(kernel="register"):
        b = fn()
    torch.cuda.synchronize()
    return a, b


def _same(a, b):
    if isinstance(a, (tuple, list)):
        for u, v in zip(a, b):
            _same(u, v)
    elif a is not None:
        assert torch.equal(a, b), "TMA and register paths differ"


@pytest.mark.parametrize("W,G,norm,gate_on,dtype", [
    (4, 1, False, False, torch.bfloat16), (4, 1, True, True, torch.bfloat16), (7, 128, True, True, torch.bfloat16),
    (3, 4, False, True, torch.float16), (7, 16, True, False, torch.float32), (5, 2, True, True, torch.bfloat16),
    (12, 8, False, True, torch.bfloat16), (4, 64, True, True, torch.bfloat16),
])
def test_training_forward(capi, W, G, norm, gate_on, dtype):
    from greta_plugin_b200.dynamic_conv import dynconv_fwd

    g = torch.Generator().manual_seed(W * 100 + G)
    lens = [1, 2, 70, 5, 300, 0, 64]
    T, D = sum(lens), 512
    x = rand(g, 1, T, D, dtype=dtype)
    w = rand(g, T, W, D // G, scale=0.5, dtype=dtype)
    gate = rand(g, 1, T, D, dtype=dtype) if gate_on else None
    cu = ragged_cu(lens)
    xd, wd, gd, cud = x.to(DEV), w.to(DEV), None if gate is None else gate.to(DEV), cu.to(DEV)
    (y1, yr1, _, _), (y2, yr2, _, _) = both(
        capi, lambda: dynconv_fwd(xd, wd, gd, cud, G, norm=norm, save_pre=True))
    _same((y1, yr1), (y2, yr2))
    yo, _ = oracle.fwd(to_np(x[0]), to_np(w), to_np(gate[0]) if gate_on else None, cu.numpy(), G, int(norm))
    assert_close(y1[0], yo, dtype)


def test_training_forward_single_sequence(capi):
    from greta_plugin_b200.dynamic_conv import dynconv_fwd

    g = torch.Generator().manual_seed(1)
    T, D, W = 777, 1024, 4
    x, w = rand(g, 1, T, D).to(DEV), rand(g, T, W, D, scale=0.5).to(DEV)
    a, b = both(capi, lambda: dynconv_fwd(x, w, None, None, 1)[0])
    _same(a, b)
    yo, _ = oracle.fwd(to_np(x[0]), to_np(w), None, None, 1, 0)
    assert_close(a[0], yo, torch.bfloat16)


@pytest.mark.parametrize("W,G,norm,gate_on", [(4, 1, False, False), (7, 128, True, True), (3, 8, True, False)])
def test_inference_from_context(capi, W, G, norm, gate_on):
    from greta_plugin_b200 import dynamic_causal_conv1d_inference

    g = torch.Generator().manual_seed(W + G)
    B, Q, D = 3, 129, 512
    ctx = rand(g, B, Q + W - 1, D).to(DEV)
    w = rand(g, B, Q, W, D // G, scale=0.5).to(DEV)
    gate = rand(g, B, Q, D).to(DEV) if gate_on else None
    a, b = both(capi, lambda: dynamic_causal_conv1d_inference(ctx, w, gate, G, norm))
    _same(a, b)
    yo = oracle.inference(to_np(ctx), to_np(w), to_np(gate), G, int(norm))
    assert_close(a, yo, torch.bfloat16)


@pytest.mark.parametrize("layout", ["DS", "SD"])
@pytest.mark.parametrize("W,G", [(4, 1), (7, 128), (4, 8), (2, 256)])
def test_packed_prefill_with_state(capi, layout, W, G):
    """Prefill-like packed batch (T > 2N) with slot history: the TMA path
    must match the register path bit for bit, including the new slot state."""
    from greta_plugin_b200 import packed_dynamic_conv_triton

    g = torch.Generator().manual_seed(W * 7 + G)
    lens = [1, 1, 2, W - 1, 90, 33, 200, 0, 5]
    slots = [3, -1, 7, 0, 11, 5, 2, 9, 4]
    init = [1, 1, 0, 1, 1, 0, 1, 0, 1]
    T, D, n_slots = sum(lens), 512, 12
    x = rand(g, T, D).to(DEV)
    w = rand(g, T, W, D // G, scale=0.5).to(DEV)
    gate = rand(g, T, D).to(DEV)
    logical = rand(g, n_slots, D, W - 1)
    starts = torch.tensor([0] + list(np.cumsum(lens)), dtype=torch.int32, device=DEV)
    sl = torch.tensor(slots, dtype=torch.int32, device=DEV)
    ini = torch.tensor(init, dtype=torch.int8, device=DEV)

    def make_state():
        if layout == "DS":
            return logical.to(DEV).contiguous()
        return logical.transpose(1, 2).contiguous().to(DEV).transpose(1, 2)

    sa, sb = make_state(), make_state()
    ya = packed_dynamic_conv_triton(x, w, gate, sa, starts, sl, ini, G)
    with capi.launch_options(kernel="register"):
        yb = packed_dynamic_conv_triton(x, w, gate, sb, starts, sl, ini, G)
    torch.cuda.synchronize()
    assert torch.equal(ya, yb)
    assert torch.equal(sa, sb)
    yo, so = oracle.packed(to_np(x), to_np(w), to_np(gate), to_np(logical), starts.cpu().numpy(), np.array(slots),
                           np.array(init), G, 2)
    assert_close(ya, yo, torch.bfloat16)
    assert np.array_equal(sa.float().cpu().numpy(), so)


@pytest.mark.parametrize("D,W,G", [(256, 4, 1), (256, 7, 128), (4096, 7, 16)])
@pytest.mark.parametrize("seed", range(6))
def test_packed_prefill_range_boundaries(capi, D, W, G, seed):
    """Prefill batches from ~100 to ~2400 tokens, so that the persistent CTAs
    get 0 to ~16 tokens each and range boundaries fall everywhere inside the
    requests: a boundary inside a request's first W-1 tokens moves to the
    request's start or to its (W-1)-th token, and offsets that do not start at
    token 0 shift every range off its nominal start (the speculative history
    rows are then not used). TMA and register paths agree bit for bit on y
    (the covered rows) and the state; with offsets from 0 both match the
    oracle; no pipeline wait times out."""
    from greta_plugin_b200 import packed_dynamic_conv_triton

    g = torch.Generator().manual_seed(1000 + seed)
    n_req = int(torch.randint(3, 20, (1,), generator=g))
    lens = torch.randint(0, 260 if seed % 2 else 40, (n_req,), generator=g).tolist()
    lens[0] = max(lens[0], 1)
    lead = 0 if seed < 3 else int(torch.randint(1, 9, (1,), generator=g))  # rows before the first request
    T = lead + sum(lens)
    if T <= 2 * n_req:  # keep it prefill-like (the TMA path)
        lens[0] += 2 * n_req
        T = lead + sum(lens)
    n_slots = n_req + 4
    slots = torch.randperm(n_slots, generator=g)[:n_req].to(torch.int32)
    slots[0] = -1
    init = (torch.rand(n_req, generator=g) > 0.2).to(torch.int8)
    x = rand(g, T, D).to(DEV)
    w = rand(g, T, W, D // G, scale=0.5).to(DEV)
    gate = rand(g, T, D).to(DEV)
    logical = rand(g, n_slots, D, W - 1)
    starts = torch.tensor([lead] + list(lead + np.cumsum(lens)), dtype=torch.int32, device=DEV)
    sl, ini = slots.to(DEV), init.to(DEV)
    outs = []
    for register_path in (False, True):
        with capi.launch_options(kernel="register" if register_path else "rows"):
            st = logical.to(DEV).clone()
            y = torch.zeros(T, D, device=DEV, dtype=torch.bfloat16)
            packed_dynamic_conv_triton(x, w, gate, st, starts, sl, ini, G, out=y)
        torch.cuda.synchronize()
        outs.append((y, st))
    (ya, sa), (yb, sb) = outs
    assert torch.equal(ya[lead:], yb[lead:])
    assert torch.equal(sa, sb)
    if lead == 0:
        yo, so = oracle.packed(to_np(x), to_np(w), to_np(gate), to_np(logical), starts.cpu().numpy(),
                               slots.numpy(), init.numpy(), G, 2)
        assert_close(ya, yo, torch.bfloat16)
        assert np.array_equal(sa.float().cpu().numpy(), so)


# --------------------------------------------------------------------------
# channel-split launches (a token range streamed by several CTAs, one per
# channel slice) and the row-streaming backward
# --------------------------------------------------------------------------
@pytest.mark.parametrize("D,W,G,norm,gate_on,dtype", [
    (4096, 7, 128, True, True, torch.bfloat16),   # 2 slices of 2048, whole filter rows
    (4096, 7, 1, False, False, torch.bfloat16),   # 2 slices, filters staged per tap
    (2048, 5, 4, True, True, torch.bfloat16),     # runtime W <= 8: 2 slices of 1024
    (1024, 12, 8, False, True, torch.float16),    # runtime W <= 16: 2 slices of 512
    (2048, 3, 16, True, False, torch.float32),
])
def test_forward_channel_split(capi, D, W, G, norm, gate_on, dtype):
    from greta_plugin_b200.dynamic_conv import dynconv_fwd

    g = torch.Generator().manual_seed(D + W + G)
    lens = [1, W - 1, 0, 3, 200, 2 * W, 90]
    T = sum(lens)
    x = rand(g, 1, T, D, dtype=dtype)
    w = rand(g, T, W, D // G, scale=0.5, dtype=dtype)
    gate = rand(g, 1, T, D, dtype=dtype) if gate_on else None
    cu = ragged_cu(lens)
    xd, wd, gd, cud = x.to(DEV), w.to(DEV), None if gate is None else gate.to(DEV), cu.to(DEV)
    (y1, yr1, _, _), (y2, yr2, _, _) = both(
        capi, lambda: dynconv_fwd(xd, wd, gd, cud, G, norm=norm, save_pre=True))
    _same((y1, yr1), (y2, yr2))
    yo, _ = oracle.fwd(to_np(x[0]), to_np(w), to_np(gate[0]) if gate_on else None, cu.numpy(), G, int(norm))
    assert_close(y1[0], yo, dtype)


@pytest.mark.parametrize("layout", ["DS", "SD"])
def test_packed_prefill_channel_split(capi, layout):
    """W = 7, G = 128 at 4096 channels: two CTAs per token range, each reading
    and writing its half of every slot."""
    from greta_plugin_b200 import packed_dynamic_conv_triton

    W, G, D, n_slots = 7, 128, 4096, 10
    g = torch.Generator().manual_seed(77)
    lens = [1, 3, 6, 7, 150, 0, 40, 9]
    slots = [3, -1, 7, 0, 8, 5, 2, 9]
    init = [1, 1, 0, 1, 1, 0, 1, 1]
    T = sum(lens)
    x = rand(g, T, D).to(DEV)
    w = rand(g, T, W, D // G, scale=0.5).to(DEV)
    gate = rand(g, T, D).to(DEV)
    logical = rand(g, n_slots, D, W - 1)
    starts = torch.tensor([0] + list(np.cumsum(lens)), dtype=torch.int32, device=DEV)
    sl = torch.tensor(slots, dtype=torch.int32, device=DEV)
    ini = torch.tensor(init, dtype=torch.int8, device=DEV)

    def make_state():
        if layout == "DS":
            return logical.to(DEV).contiguous()
        return logical.transpose(1, 2).contiguous().to(DEV).transpose(1, 2)

    sa, sb = make_state(), make_state()
    ya = packed_dynamic_conv_triton(x, w, gate, sa, starts, sl, ini, G)
    with capi.launch_options(kernel="register"):
        yb = packed_dynamic_conv_triton(x, w, gate, sb, starts, sl, ini, G)
    torch.cuda.synchronize()
    assert torch.equal(ya, yb)
    assert torch.equal(sa, sb)
    yo, so = oracle.packed(to_np(x), to_np(w), to_np(gate), to_np(logical), starts.cpu().numpy(), np.array(slots),
                           np.array(init), G, 2)
    assert_close(ya, yo, torch.bfloat16)
    assert np.array_equal(sa.float().cpu().numpy(), so)


def test_inference_channel_split(capi):
    from greta_plugin_b200 import dynamic_causal_conv1d_inference

    W, G, D, B, Q = 7, 128, 2048, 2, 300
    g = torch.Generator().manual_seed(5)
    ctx = rand(g, B, Q + W - 1, D).to(DEV)
    w = rand(g, B, Q, W, D // G, scale=0.5).to(DEV)
    gate = rand(g, B, Q, D).to(DEV)
    a, b = both(capi, lambda: dynamic_causal_conv1d_inference(ctx, w, gate, G, True))
    _same(a, b)
    yo = oracle.inference(to_np(ctx), to_np(w), to_np(gate), G, 1)
    assert_close(a, yo, torch.bfloat16)


@pytest.mark.parametrize("D,W,G,norm,gate_on,dtype,lens", [
    (512, 4, 1, False, False, torch.bfloat16, [1, 2, 3, 300, 0, 64, 5]),
    (512, 4, 64, True, True, torch.bfloat16, [1, 2, 3, 300, 0, 64, 5]),
    (4096, 4, 1, False, False, torch.bfloat16, [700, 3, 1, 300]),      # 2 slices, filters per tap
    (4096, 4, 1, True, True, torch.bfloat16, [257, 2, 400]),
    (2048, 7, 128, True, True, torch.bfloat16, [1, 6, 7, 8, 5000, 0]),  # 1 slice, producer in warp 0
    (4096, 7, 128, False, True, torch.bfloat16, [3000, 1, 999]),         # 2 slices, producer in warp 0
    # many short requests of odd and even lengths: tokens in pairs and alone
    (2048, 7, 64, True, True, torch.bfloat16, [2, 3, 1, 4, 9, 10, 11, 2, 1, 13, 40, 7, 8, 0, 5, 6, 300]),
    (2048, 7, 128, False, True, torch.bfloat16, [1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12, 13, 14, 15, 160]),
    (4096, 7, 8, True, False, torch.bfloat16, [2000, 50]),               # the same, filters per tap
    (2048, 7, 2, False, False, torch.bfloat16, [700, 5, 300]),           # 2 slices of 1024, producer warp
    (1024, 7, 16, False, True, torch.float16, [30, 31, 200]),
    (768, 3, 2, True, False, torch.float32, [5, 100, 1, 2]),           # 768 = 3 x 256: one slice
    (1024, 2, 4, False, True, torch.bfloat16, [1, 1, 1, 1, 90]),
    (512, 8, 8, True, True, torch.bfloat16, [9, 8, 7, 150]),
    (256, 5, 128, True, True, torch.bfloat16, [4, 5, 6, 60]),
    (512, 3, 128, True, True, torch.bfloat16, [3, 70, 1]),             # runtime W, 16 lanes per group
    (512, 4, 32, False, True, torch.bfloat16, [2, 90]),                 # 4 lanes per group
    (512, 4, 1, True, False, torch.bfloat16, [1, 2, 3]),                # fewer tokens than SMs
])
def test_training_backward(capi, D, W, G, norm, gate_on, dtype, lens):
    """Row-streaming backward against the register-staged backward (bit for
    bit) and the oracle, over ragged packs with empty and short sequences."""
    from greta_plugin_b200.dynamic_conv import dynconv_bwd, dynconv_fwd

    g = torch.Generator().manual_seed(D * 3 + W * 5 + G)
    T = sum(lens)
    x = rand(g, 1, T, D, dtype=dtype)
    w = rand(g, T, W, D // G, scale=(1.0 / W) ** 0.5, dtype=dtype)
    gate = rand(g, 1, T, D, dtype=dtype) if gate_on else None
    dout = rand(g, 1, T, D, dtype=dtype)
    cu = ragged_cu(lens)
    xd, wd, dd, cud = x.to(DEV), w.to(DEV), dout.to(DEV), cu.to(DEV)
    gd = gate.to(DEV) if gate_on else None
    _, yr, _, _ = dynconv_fwd(xd, wd, gd, cud, G, norm=norm, save_pre=True)
    a, b = both(capi, lambda: dynconv_bwd(xd, wd, gd, yr, dd, cud, G, norm, 1e-6, 64, None))
    _same(a, b)
    dx, dw, dg = a
    gn = to_np(gate[0]) if gate_on else None
    dxo, dwo, dgo = oracle.bwd(to_np(x[0]), to_np(w), gn, to_np(dout[0]), cu.numpy(), G, int(norm),
                               yr=to_np(yr[0]) if norm else None)
    assert_close(dx[0], dxo, dtype)
    assert_close(dw, dwo, dtype)
    if gate_on:
        assert_close(dg[0], dgo, dtype)


def test_training_backward_single_sequence(capi):
    from greta_plugin_b200.dynamic_conv import dynconv_bwd

    g = torch.Generator().manual_seed(11)
    T, D, W = 1000, 4096, 4
    x, w = rand(g, 1, T, D).to(DEV), rand(g, T, W, D, scale=0.5).to(DEV)
    dout = rand(g, 1, T, D).to(DEV)
    a, b = both(capi, lambda: dynconv_bwd(x, w, None, None, dout, None, 1, False, 1e-6, 64, None))
    _same(a, b)
    dxo, dwo, _ = oracle.bwd(to_np(x[0]), to_np(w), None, to_np(dout[0]), None, 1, 0)
    assert_close(a[0][0], dxo, torch.bfloat16)
    assert_close(a[1], dwo, torch.bfloat16)


def test_pipeline_wait_runs_out_and_the_kernel_returns(capi):
    """A bounded pipeline wait that runs out: with the test hook, consumer warp
    0 of CTA 0 keeps the first stage it used, so CTA 0's producer waits for a
    release that never comes. Its wait (2^14 polls) runs out, it records the
    timeout bit and returns; CTA 0's consumers then wait for a stage that is
    never filled and return the same way. Every bulk copy that was issued has
    landed by then (the consumers waited for each), nothing faults, the call
    returns, the error word reports the timeout, and the context runs normal
    launches with correct results afterwards. 4096 tokens x 4096 channels:
    each of the CTAs streams ~27 one-token stages through a ring of 5, so the
    refill is reached."""
    from greta_plugin_b200.dynamic_conv import dynconv_fwd

    g = torch.Generator().manual_seed(77)
    T, D, W = 4096, 4096, 4
    x = rand(g, 1, T, D).to(DEV)
    w = rand(g, T, W, D, scale=0.5).to(DEV)
    capi.device_errors(clear=True)
    with capi.launch_options(wait_limit_log2=14, test_withhold_release=True):
        y_bad, _, _, _ = dynconv_fwd(x, w, None, None, 1)
    torch.cuda.synchronize()
    bits = capi.device_errors(clear=True)
    assert bits & capi.ERR_BIT_TIMEOUT, f"expected the timeout bit, got {bits:#x}"
    # the context is intact: a normal launch afterwards is correct and clean
    y, _, _, _ = dynconv_fwd(x, w, None, None, 1)
    torch.cuda.synchronize()
    assert capi.device_errors(clear=True) == 0
    yo, _ = oracle.fwd(to_np(x[0]), to_np(w), None, None, 1, 0)
    assert_close(y[0], yo, torch.bfloat16)
    # the other CTAs of the stopped launch finished their ranges: the last
    # token rows (far from CTA 0's range) match
    assert torch.equal(y_bad[0, -64:], y[0, -64:])
    # the checked vLLM entry point turns the bit into an exception
    from greta_plugin_b200.vllm_conv import packed_dynamic_conv_checked

    starts = torch.tensor([0, T], dtype=torch.int32, device=DEV)
    state = torch.zeros(1, D, W - 1, dtype=torch.bfloat16, device=DEV)
    one = torch.ones(1, dtype=torch.int8, device=DEV)
    slot = torch.zeros(1, dtype=torch.int32, device=DEV)
    with capi.launch_options(kernel="rows", wait_limit_log2=14, test_withhold_release=True):
        with pytest.raises(capi.GretaKernelError, match="timed out"):
            packed_dynamic_conv_checked(x[0], w, None, state, starts, slot, one, 1, norm=False)
    assert capi.device_errors(clear=True) == 0
