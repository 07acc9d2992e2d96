"""vLLM packed path (greta_vllm/triton_conv.py) on the GPU vs the CPU oracle:
chunked prefill and decode with cache-slot history, padding slots (-1),
has_initial off, chunks shorter than W-1, both vLLM state orientations and a
generic strided state, the benchmark-sized prefill and decode configurations,
CUDA-graph capture, and out-of-range slot detection. Output within
rtol = atol = 1e-2 (bf16); conv state bit-exact."""
import numpy as np
import pytest
import torch

from gpu_helpers import DEV, assert_close, bf16_bits, rand, to_np
from oracle import oracle

pytestmark = pytest.mark.gpu


def make_batch(lengths, slots, init, n_slots, D, W, G, dtype, seed, gate_on=True, layout="DS"):
    g = torch.Generator().manual_seed(seed)
    T = int(sum(lengths))
    x = rand(g, T, D, dtype=dtype)
    w = rand(g, T, W, D // G, scale=(1.0 / W) ** 0.5, dtype=dtype)
    gate = rand(g, T, D, dtype=dtype) if gate_on else None
    logical = rand(g, n_slots, D, W - 1, dtype=dtype)
    starts = torch.tensor([0] + list(np.cumsum(lengths)), dtype=torch.int32)
    if layout == "DS":
        state = logical.to(DEV).contiguous()
    elif layout == "SD":  # vLLM stores [slots, W-1, D] and hands over the transposed view
        state = logical.transpose(1, 2).contiguous().to(DEV).transpose(1, 2)
    else:  # padded slot stride: generic addressing
        big = torch.zeros(n_slots, D * (W - 1) + 5, dtype=dtype)
        big[:, : D * (W - 1)] = logical.reshape(n_slots, -1)
        state = big.to(DEV).as_strided((n_slots, D, W - 1), (D * (W - 1) + 5, W - 1, 1))
    return dict(x=x, w=w, gate=gate, logical=logical, starts=starts, slots=torch.tensor(slots, dtype=torch.int32),
                init=torch.tensor(init, dtype=torch.int8), state=state, G=G)


def run_and_check(b, norm=True, dtype=torch.bfloat16):
    from greta_plugin_b200 import packed_dynamic_conv_triton

    st_before = b["state"].clone()
    out = packed_dynamic_conv_triton(b["x"].to(DEV), b["w"].to(DEV), None if b["gate"] is None else b["gate"].to(DEV),
                                     b["state"], b["starts"].to(DEV), b["slots"].to(DEV), b["init"].to(DEV), b["G"],
                                     norm=norm, eps=1e-6)
    yo, so = oracle.packed(to_np(b["x"]), to_np(b["w"]), to_np(b["gate"]), to_np(b["logical"]), b["starts"].numpy(),
                           b["slots"].numpy(), b["init"].numpy(), b["G"], 2 if norm else 0)
    assert_close(out, yo, dtype)
    got_state = b["state"].float().cpu().numpy()
    assert np.array_equal(got_state, so), "conv state must be bit-exact"
    # slots that no request names are untouched
    named = set(int(s) for s in b["slots"].tolist() if s >= 0)
    for s in range(b["state"].shape[0]):
        if s not in named:
            assert torch.equal(b["state"][s], st_before[s])
    return out


@pytest.mark.parametrize("layout", ["DS", "SD", "generic"])
@pytest.mark.parametrize("W,G", [(4, 1), (4, 8), (7, 128), (3, 2), (5, 16), (2, 256)])
def test_mixed_batches(layout, W, G):
    lengths = [1, 1, 1, 1, 2, W - 1, 40, 3, 129]
    slots = [3, -1, 7, 0, 11, 5, 2, -1, 9]
    init = [1, 1, 0, 1, 1, 1, 0, 1, 1]
    b = make_batch(lengths, slots, init, 12, 256, W, G, torch.bfloat16, seed=W * 31 + G, layout=layout)
    run_and_check(b)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("norm", [True, False])
def test_dtypes_and_norm(dtype, norm):
    b = make_batch([1, 1, 5, 60], [0, 1, 2, 3], [1, 0, 1, 1], 4, 128, 4, 4, dtype, seed=5)
    run_and_check(b, norm=norm, dtype=dtype)


@pytest.mark.parametrize("lengths", [[1, 3, 60], [1, 1, 1]])  # row-streaming and register kernels
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_stable_norm_huge_values(dtype, lengths):
    """The overflow-safe norm of the vLLM path on inputs whose conv outputs are
    ~3e37 (their squares overflow fp32, some group maxima exceed 2^126): finite
    and within tolerance of the oracle."""
    b = make_batch(lengths, [0, -1, 2], [1, 1, 1], 3, 256, 4, 4, dtype, seed=17)
    for k in ("x", "logical"):
        b[k] = (b[k].float() * 3e37).to(dtype)
    b["state"].copy_(b["logical"].to(DEV))
    out = run_and_check(b, norm=True, dtype=dtype)
    assert torch.isfinite(out.float()).all()


@pytest.mark.parametrize("lengths", [[1, 3, 60], [1, 1, 1]])  # row-streaming and decode kernels
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_stable_norm_group_max_at_2_pow_60(dtype, lengths):
    """A 256-channel group whose conv outputs are all exactly +-2^60: 256 squares
    of 2^60 sum to 2^128, which is inf in fp32, so the one-pass sum of squares
    must not be used there (the rescaled form gives +-1). Rows just below
    (2^60 (1 - 2^-8)) and just above (2^60 (1 + 2^-7)) the bound are checked
    too. The filters pass the current input through unchanged (tap W-1 = 1,
    the others 0), so y equals x exactly."""
    D, W, G = 256, 4, 256
    T = sum(lengths)
    g = torch.Generator().manual_seed(60)
    mags = torch.tensor([2.0 ** 60, 2.0 ** 60 * (1 - 2 ** -8), 2.0 ** 60 * (1 + 2 ** -7)], dtype=torch.float64)
    sign = torch.where(torch.rand(T, D, generator=g) < 0.5, -1.0, 1.0).double()
    x = (sign * mags[torch.arange(T) % 3][:, None]).to(dtype)
    assert torch.equal(x.double().abs()[0], torch.full((D,), 2.0 ** 60, dtype=torch.float64))
    w = torch.zeros(T, W, D // G, dtype=dtype)
    w[:, W - 1] = 1.0
    b = make_batch(lengths, [0, -1, 2], [0, 1, 0], 3, D, W, G, dtype, seed=61, gate_on=False)
    b["x"], b["w"] = x, w
    out = run_and_check(b, norm=True, dtype=dtype)
    o = out.float().cpu()
    assert torch.isfinite(o).all()
    # every row's group is one magnitude, so the normalised row is +-1
    torch.testing.assert_close(o, sign.float(), rtol=0, atol=1e-2)


@pytest.mark.parametrize("layout", ["DS", "SD", "generic"])
@pytest.mark.parametrize("D,W,G", [(4096, 4, 512), (2048, 7, 1024), (4096, 7, 4096), (1024, 3, 512), (2048, 2, 2048)])
def test_wide_groups(layout, D, W, G):
    """Groups wider than 256 channels (the reference's supports() accepts any
    power of two dividing D, greta_vllm/triton_conv.py:119-121): one CTA per
    group; mixed decodes and prefill chunks, padding slots, has_initial off,
    requests shorter than W-1 and longer than a chunk."""
    lengths = [1, 1, 1, 2, W - 1, 0, 17, 40]
    slots = [3, -1, 7, 0, 11, 1, 5, 9]
    init = [1, 1, 0, 1, 1, 0, 1, 0]
    b = make_batch(lengths, slots, init, 12, D, W, G, torch.bfloat16, seed=D + W + G, layout=layout)
    run_and_check(b)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
@pytest.mark.parametrize("norm,gate_on", [(True, False), (False, True), (False, False)])
def test_wide_groups_dtypes_norm_gate(dtype, norm, gate_on):
    b = make_batch([1, 1, 5, 60], [0, 1, 2, 3], [1, 0, 1, 1], 4, 2048, 4, 512, dtype, seed=9, gate_on=gate_on)
    run_and_check(b, norm=norm, dtype=dtype)


@pytest.mark.parametrize("scale", [3e37, 2.0 ** 47, 2.0 ** 48, 2.0 ** 49])
def test_wide_groups_stable_norm_large_values(scale):
    """The overflow-safe norm of a 1024-channel group at and around its
    one-pass bound (max|y| < 2^48) and near the fp32 limit: finite and within
    tolerance of the oracle."""
    b = make_batch([1, 3, 60], [0, -1, 2], [1, 1, 1], 3, 2048, 4, 1024, torch.float32, seed=19)
    for k in ("x", "logical"):
        b[k] = (b[k].float() * scale).float()
    b["state"].copy_(b["logical"].to(DEV))
    out = run_and_check(b, norm=True, dtype=torch.float32)
    assert torch.isfinite(out.float()).all()


def test_prefill_config_varlen_1024():
    """Varlen chunked prefill: 8 sequences with lengths ~U[32, 256] (sum <= 1024),
    C=4096, K=4, state [64, 4096, 3] ~ N(0,1) read from 8 distinct slots."""
    g = torch.Generator().manual_seed(0)
    while True:
        lengths = torch.randint(32, 257, (8,), generator=g).tolist()
        if sum(lengths) <= 1024:
            break
    slots = torch.randperm(64, generator=g)[:8].tolist()
    b = make_batch(lengths, slots, [1] * 8, 64, 4096, 4, 1, torch.bfloat16, seed=1, gate_on=False)
    run_and_check(b, norm=False)


def test_decode_config_256_of_1024_slots():
    """Decode: 256 requests of one token, C=4096, K=4, state [1024, 4096, 3],
    distinct slots with 10% set to -1."""
    g = torch.Generator().manual_seed(0)
    slots = torch.randperm(1024, generator=g)[:256]
    pad = torch.randperm(256, generator=g)[:26]
    slots[pad] = -1
    b = make_batch([1] * 256, slots.tolist(), [1] * 256, 1024, 4096, 4, 1, torch.bfloat16, seed=2, gate_on=False)
    run_and_check(b, norm=False)


def test_repeated_decode_steps_shift_state():
    """Ten decode steps in a row equal ten oracle steps (state carried)."""
    from greta_plugin_b200 import packed_dynamic_conv_triton

    D, W, G, N = 256, 4, 8, 16
    g = torch.Generator().manual_seed(9)
    logical = rand(g, 32, D, W - 1)
    state = logical.to(DEV).clone()
    ostate = to_np(logical)
    slots = torch.randperm(32, generator=g)[:N].to(torch.int32)
    starts = torch.arange(N + 1, dtype=torch.int32)
    init = torch.ones(N, dtype=torch.int8)
    for step in range(10):
        x = rand(g, N, D)
        w = rand(g, N, W, D // G, scale=0.5)
        gate = rand(g, N, D)
        y = packed_dynamic_conv_triton(x.to(DEV), w.to(DEV), gate.to(DEV), state, starts.to(DEV), slots.to(DEV),
                                       init.to(DEV), G)
        yo, ostate = oracle.packed(to_np(x), to_np(w), to_np(gate), ostate, starts.numpy(), slots.numpy(),
                                   init.numpy(), G, 2)
        assert_close(y, yo, torch.bfloat16)
        assert np.array_equal(state.float().cpu().numpy(), ostate)


def test_zero_length_requests_and_empty_batch():
    from greta_plugin_b200 import packed_dynamic_conv_triton

    b = make_batch([0, 3, 0, 5], [1, 2, 3, 0], [1, 1, 0, 1], 4, 64, 4, 4, torch.bfloat16, seed=4)
    run_and_check(b)
    # T == 0 returns immediately (greta_vllm/triton_conv.py:142-143): state untouched
    st = b["state"].clone()
    out = packed_dynamic_conv_triton(torch.zeros(0, 64, device=DEV, dtype=torch.bfloat16),
                                     torch.zeros(0, 4, 16, device=DEV, dtype=torch.bfloat16), None, b["state"],
                                     torch.zeros(1, dtype=torch.int32, device=DEV),
                                     torch.zeros(0, dtype=torch.int32, device=DEV),
                                     torch.zeros(0, dtype=torch.int8, device=DEV), 4)
    assert out.shape == (0, 64) and torch.equal(st, b["state"])


def test_out_argument_is_filled_in_place():
    from greta_plugin_b200 import packed_dynamic_conv_triton

    b = make_batch([1, 7], [0, 1], [1, 1], 2, 64, 4, 1, torch.bfloat16, seed=6)
    out_full = torch.full((12, 64), 7.0, device=DEV, dtype=torch.bfloat16)
    out = packed_dynamic_conv_triton(b["x"].to(DEV), b["w"].to(DEV), b["gate"].to(DEV), b["state"],
                                     b["starts"].to(DEV), b["slots"].to(DEV), b["init"].to(DEV), 1,
                                     out=out_full[:8])
    assert out.data_ptr() == out_full.data_ptr()
    assert torch.all(out_full[8:] == 7.0)


def test_cuda_graph_capture_of_decode_step():
    """The decode launch allocates nothing and syncs nothing: capture + replay."""
    from greta_plugin_b200 import packed_dynamic_conv_triton

    D, W, G, N = 512, 4, 1, 64
    g = torch.Generator().manual_seed(11)
    x = rand(g, N, D).to(DEV)
    w = rand(g, N, W, D // G, scale=0.5).to(DEV)
    logical = rand(g, 128, D, W - 1)
    state = logical.to(DEV).clone()
    slots = torch.randperm(128, generator=g)[:N].to(torch.int32).to(DEV)
    starts = torch.arange(N + 1, dtype=torch.int32, device=DEV)
    init = torch.ones(N, dtype=torch.int8, device=DEV)
    out = torch.empty_like(x)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):  # warm-up outside capture (library load)
        packed_dynamic_conv_triton(x, w, None, state.clone(), starts, slots, init, G, out=out)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        packed_dynamic_conv_triton(x, w, None, state, starts, slots, init, G, out=out)
    state.copy_(logical.to(DEV))
    ostate = to_np(logical)
    for _ in range(3):
        graph.replay()
        yo, ostate = oracle.packed(to_np(x), to_np(w), None, ostate, starts.cpu().numpy(), slots.cpu().numpy(),
                                   init.cpu().numpy(), G, 2)
        torch.cuda.synchronize()
        assert_close(out, yo, torch.bfloat16)
        assert np.array_equal(state.float().cpu().numpy(), ostate)
    del graph


def test_out_of_range_slot_is_skipped_and_reported():
    from greta_plugin_b200.vllm_conv import packed_dynamic_conv_checked

    b = make_batch([1, 4], [1, 99], [1, 1], 4, 64, 4, 1, torch.bfloat16, seed=12)
    st = b["state"].clone()
    with pytest.raises(IndexError):
        packed_dynamic_conv_checked(b["x"].to(DEV), b["w"].to(DEV), b["gate"].to(DEV), b["state"],
                                    b["starts"].to(DEV), b["slots"].to(DEV), b["init"].to(DEV), 1)
    # request 1's slot was out of range: nothing but slot 1 changed
    for s in (0, 2, 3):
        assert torch.equal(st[s], b["state"][s])


def test_unsupported_group_raises_reference_error():
    from greta_plugin_b200 import packed_dynamic_conv_triton, supports

    assert supports(128, 2048) and not supports(3, 48) and supports(512, 2048) and not supports(4096, 2048)
    b = make_batch([2], [0], [1], 1, 48, 4, 1, torch.bfloat16, seed=1)
    with pytest.raises(ValueError, match="power-of-two group size"):
        packed_dynamic_conv_triton(b["x"].to(DEV), torch.zeros(2, 4, 16, device=DEV, dtype=torch.bfloat16), None,
                                   b["state"], b["starts"].to(DEV), b["slots"].to(DEV), b["init"].to(DEV), 3)


def test_state_bits_are_copies_of_inputs():
    """Write-back moves data only: every new slot element is an input element."""
    b = make_batch([5, 9], [0, 1], [0, 1], 2, 64, 4, 1, torch.bfloat16, seed=13)
    run_and_check(b)
    xb = bf16_bits(b["x"])
    sb = bf16_bits(b["state"].cpu())
    assert np.array_equal(sb[0], xb[2:5].T)
    assert np.array_equal(sb[1], xb[11:14].T)
