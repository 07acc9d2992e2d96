"""Prefill-like vLLM packed batches on the row-streaming kernel (the default
for them) against the register-staged kernel (the same arithmetic:
bit-identical outputs and states) and the oracle
(greta_vllm/triton_conv.py:28-116 semantics), on the cases where a request's
first W-1 tokens (its head region, the only tokens that read the cache slot)
meet a CTA's range boundary: requests starting at every offset of 8-token
blocks, requests shorter than W-1, empty requests (in the middle, first, and
at offset T), tokens outside every request, padding slots, has_initial off,
every state layout, norm kinds, gate, dtypes, and many requests."""
import numpy as np
import pytest
import torch

from gpu_helpers import DEV, assert_close, rand, to_np
from oracle import oracle

pytestmark = pytest.mark.gpu


def batch(lengths, slots, init, n_slots, D, W, G, dtype, seed, gate_on=True, layout="DS", lead=0, tail=0):
    """A packed batch of `lengths` starting at token `lead`, with `tail` unused
    tokens after the last request."""
    g = torch.Generator().manual_seed(seed)
    T = lead + int(sum(lengths)) + tail
    x = rand(g, T, D, dtype=dtype)
    w = rand(g, T, W, D // G, scale=(1.0 / W) ** 0.5, dtype=dtype)
    gate = rand(g, T, D, dtype=dtype) if gate_on else None
    logical = rand(g, n_slots, D, W - 1, dtype=dtype)
    starts = torch.tensor([lead] + list(lead + np.cumsum(lengths)), dtype=torch.int32)
    return dict(x=x, w=w, gate=gate, logical=logical, starts=starts, slots=torch.tensor(slots, dtype=torch.int32),
                init=torch.tensor(init, dtype=torch.int8), G=G, layout=layout, lead=lead, T=T)


def state_of(b):
    logical = b["logical"]
    if b["layout"] == "DS":
        return logical.to(DEV).contiguous()
    if b["layout"] == "SD":
        return logical.transpose(1, 2).contiguous().to(DEV).transpose(1, 2)
    n, D, H = logical.shape
    big = torch.zeros(n, D * H + 5, dtype=logical.dtype)
    big[:, : D * H] = logical.reshape(n, -1)
    return big.to(DEV).as_strided((n, D, H), (D * H + 5, H, 1))


def run(b, kernel, norm, out_fill=0.0):
    from greta_plugin_b200 import _capi, packed_dynamic_conv_triton

    state = state_of(b)
    y = torch.full(b["x"].shape, out_fill, dtype=b["x"].dtype, device=DEV)
    with _capi.launch_options(kernel=kernel):
        packed_dynamic_conv_triton(b["x"].to(DEV), b["w"].to(DEV), None if b["gate"] is None else b["gate"].to(DEV),
                                   state, b["starts"].to(DEV), b["slots"].to(DEV), b["init"].to(DEV), b["G"],
                                   norm=norm, eps=1e-6, out=y)
    torch.cuda.synchronize()
    return y, state


def check(b, norm=True, dtype=torch.bfloat16, kernels=("rows", "register")):
    outs = {k: run(b, k, norm) for k in kernels}
    yf, sf = outs["rows"]
    for k, (y, s) in outs.items():
        assert torch.equal(y.view(torch.int16 if y.element_size() == 2 else torch.int32),
                           yf.view(torch.int16 if yf.element_size() == 2 else torch.int32)), f"rows != {k}: y"
        assert torch.equal(s.contiguous().view(torch.int16 if s.element_size() == 2 else torch.int32),
                           sf.contiguous().view(torch.int16 if sf.element_size() == 2 else torch.int32)), \
            f"rows != {k}: state"
    lead, T = b["lead"], b["T"]
    end = int(b["starts"][-1])
    yo, so = oracle.packed(to_np(b["x"]), to_np(b["w"]), to_np(b["gate"]), to_np(b["logical"]),
                           b["starts"].numpy(), b["slots"].numpy(), b["init"].numpy(), b["G"], 2 if norm else 0)
    assert_close(yf[lead:end], yo[lead:end], dtype)
    assert np.array_equal(sf.float().cpu().numpy(), so), "conv state must be bit-exact"
    # tokens outside every request are not written
    if lead or end < T:
        y_again, _ = run(b, "rows", norm, out_fill=7.0)
        assert (y_again[:lead].float() == 7.0).all() and (y_again[end:].float() == 7.0).all()


@pytest.mark.parametrize("W", [2, 3, 4, 5, 7, 8])
@pytest.mark.parametrize("first", range(8))
def test_head_region_at_every_cta_offset(W, first):
    """Requests start at every offset of an 8-token CTA range, so their first
    W-1 tokens cross the CTA boundary in every way."""
    lengths = [first + 8, 11, W - 1 if W > 1 else 1, 1, 9, 17, 3]
    slots = [3, 0, 7, 11, -1, 5, 2]
    init = [1, 1, 0, 1, 1, 1, 1]
    b = batch(lengths, slots, init, 12, 256, W, 8, torch.bfloat16, seed=100 * W + first)
    check(b)


@pytest.mark.parametrize("layout", ["DS", "SD", "generic"])
@pytest.mark.parametrize("W,G", [(4, 1), (7, 128), (4, 8), (3, 2), (5, 16), (2, 256), (7, 1), (6, 4)])
def test_layouts_and_groups(layout, W, G):
    lengths = [40, 1, 2, W - 1, 0, 23, 3, 129, 0]
    slots = [3, -1, 7, 0, 11, 5, 2, 9, 1]
    init = [1, 1, 0, 1, 0, 1, 1, 0, 0]
    b = batch(lengths, slots, init, 12, 512, W, G, torch.bfloat16, seed=W * 31 + G, layout=layout)
    check(b)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("norm,gate_on", [(True, True), (True, False), (False, True), (False, False)])
def test_dtypes_norm_gate(dtype, norm, gate_on):
    b = batch([17, 1, 5, 60, 2], [0, 1, 2, 3, 4], [1, 0, 1, 1, 1], 5, 256, 4, 4, dtype, seed=5, gate_on=gate_on)
    check(b, norm=norm, dtype=dtype)


def test_empty_requests_first_middle_and_at_the_end():
    """An empty request with history keeps its slot, without history clears it;
    at offset 0, in the middle, and at offset T (after the last token)."""
    lengths = [0, 12, 0, 0, 9, 14, 0]
    slots = [4, 0, 5, -1, 1, 2, 6]
    init = [0, 1, 1, 0, 1, 0, 1]
    b = batch(lengths, slots, init, 8, 256, 4, 1, torch.bfloat16, seed=9)
    check(b)
    lengths = [11, 6, 0, 0]
    b = batch(lengths, [0, 1, 2, 3], [1, 1, 0, 1], 4, 256, 7, 128, torch.bfloat16, seed=10)
    check(b)


@pytest.mark.parametrize("lead,tail", [(5, 0), (0, 6), (9, 13)])
def test_tokens_outside_every_request(lead, tail):
    b = batch([20, 3, 31], [2, 0, 1], [1, 1, 1], 3, 256, 4, 1, torch.bfloat16, seed=11, lead=lead, tail=tail)
    check(b)


def test_many_requests():
    """512 and 2048 requests (the row-streaming kernel's shared-memory limit),
    lengths 1..5, one padding slot in ten; 2049 runs on the register kernel."""
    rng = np.random.default_rng(3)
    for n in (512, 2048, 2049):
        lengths = list(rng.integers(1, 6, n))
        slots = [i if i % 10 else -1 for i in range(n)]
        init = list(rng.integers(0, 2, n))
        b = batch(lengths, slots, init, n, 256, 4, 1, torch.bfloat16, seed=12)
        check(b)


def test_headline_prefill_shape():
    """The benchmark's prefill: 8 requests of 32..256 tokens (898), C=4096, K=4,
    state [64, 4096, 3]."""
    lengths = [179, 87, 54, 114, 71, 90, 148, 155]
    b = batch(lengths, [5, 17, 2, 40, 63, 0, 9, 33], [1] * 8, 64, 4096, 4, 1, torch.bfloat16, seed=13,
              gate_on=False)
    check(b, norm=False)


def test_greta_layer_prefill_shape():
    lengths = [179, 87, 54, 114, 71, 90, 148, 155]
    b = batch(lengths, [5, 17, 2, 40, 63, 0, 9, 33], [1, 0, 1, 1, 1, 1, 0, 1], 64, 2048, 7, 128,
              torch.bfloat16, seed=14, layout="SD")
    check(b)
