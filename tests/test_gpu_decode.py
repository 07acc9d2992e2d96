"""Decode-like vLLM packed batches (at most 2 tokens per request on average,
greta_vllm/triton_conv.py:28-116 with the decodes first, greta_vllm/conv.py:84-94)
on the decode kernel vs the CPU oracle: one-token requests with padding slots
(-1), has_initial off, empty requests, requests longer than one chunk (later
chunks found on the device), both vLLM state orientations and a generic
strided state (served by the register kernel), W = 4 and 7 (and W = 5, the
register kernel), every group-vector width, both norms and the gate.
Output within rtol = atol = 1e-2 (16-bit), conv state bit-exact; and the
decode kernel is bit-identical to the register kernel it replaces for these
batches."""
import numpy as np
import pytest
import torch

from gpu_helpers import DEV
from test_gpu_packed import make_batch, run_and_check

pytestmark = pytest.mark.gpu



def decode_batch(n_req, n_slots, seed, extra=None):
    """n_req one-token requests on distinct slots, ~10% padding, a few with
    has_initial = 0; `extra` appends (length, slot, init) requests."""
    g = torch.Generator().manual_seed(seed)
    slots = torch.randperm(n_slots, generator=g)[:n_req].tolist()
    for i in range(0, n_req, 10):
        slots[i] = -1
    init = [0 if i % 7 == 3 else 1 for i in range(n_req)]
    lengths = [1] * n_req
    for (L, s, f) in extra or []:
        lengths.append(L)
        slots.append(s)
        init.append(f)
    return lengths, slots, init


@pytest.mark.parametrize("layout", ["DS", "SD", "generic"])
@pytest.mark.parametrize("W,G", [(4, 1), (4, 2), (4, 8), (7, 16), (7, 128), (5, 4)])
@pytest.mark.parametrize("gate", [True, False])
def test_decode_batches(layout, W, G, gate):
    lengths, slots, init = decode_batch(40, 64, seed=W * 7 + G)
    b = make_batch(lengths, slots, init, 64, 256, W, G, torch.bfloat16, seed=G + W, gate_on=gate, layout=layout)
    run_and_check(b, norm=True)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("norm", [True, False])
def test_decode_dtypes(dtype, norm):
    lengths, slots, init = decode_batch(24, 32, seed=3)
    b = make_batch(lengths, slots, init, 32, 512, 4, 1, dtype, seed=8, gate_on=True)
    run_and_check(b, norm=norm, dtype=dtype)


@pytest.mark.parametrize("W", [4, 7])
@pytest.mark.parametrize("layout", ["DS", "SD"])
def test_mixed_lengths_in_decode_batch(W, layout):
    """A decode-like batch (T <= 2 * requests) that holds empty requests,
    requests shorter than W-1, and requests spanning several 8-token chunks
    (first chunk on the request's own CTA row, the rest found by the scan;
    the new taps of a long request come from its last W-1 inputs)."""
    extra = [(0, 100, 0), (0, 101, 1), (2, 102, 1), (W - 1, 103, 0), (9, 104, 1), (37, 105, 1), (17, -1, 1),
             (8, 106, 1)]
    lengths, slots, init = decode_batch(64, 100, seed=W, extra=extra)
    assert sum(lengths) <= 2 * len(lengths)
    b = make_batch(lengths, slots, init, 112, 256, W, 16, torch.bfloat16, seed=W + 1, layout=layout)
    run_and_check(b, norm=True)


def test_decode_kernel_bit_identical_to_register_kernel():
    """The decode kernel and the register kernel (forced by a 256-thread CTA
    shape, which the decode kernel does not take) give the same bits for y and
    the state on the same decode-like batch."""
    from greta_plugin_b200 import _capi, packed_dynamic_conv_triton

    extra = [(0, 90, 0), (2, 91, 1), (21, 92, 1)]
    for W, G in ((4, 1), (7, 128), (4, 8)):
        lengths, slots, init = decode_batch(80, 90, seed=W + G, extra=extra)
        b = make_batch(lengths, slots, init, 96, 1024, W, G, torch.bfloat16, seed=21, gate_on=True)
        outs = []
        for shape in ((0, 0, 0), (256, 1, 8)):
            with _capi.launch_options(block_x=shape[0], block_y=shape[1], tokens=shape[2]):
                state = b["state"].clone()
                y = packed_dynamic_conv_triton(b["x"].to(DEV), b["w"].to(DEV), b["gate"].to(DEV), state,
                                               b["starts"].to(DEV), b["slots"].to(DEV), b["init"].to(DEV), G,
                                               norm=True, eps=1e-6)
                outs.append((y, state))
        assert torch.equal(outs[0][0].view(torch.int16), outs[1][0].view(torch.int16))
        assert torch.equal(outs[0][1].view(torch.int16), outs[1][1].view(torch.int16))


def test_decode_config_greta_layer():
    """Greta's layer shape in a decode step: D=2048, W=7, G=128, stable norm and
    gate, 256 requests of a [1024, 2048, 6] state, 10% padding."""
    g = torch.Generator().manual_seed(0)
    slots = torch.randperm(1024, generator=g)[:256]
    slots[torch.randperm(256, generator=g)[:26]] = -1
    b = make_batch([1] * 256, slots.tolist(), [1] * 256, 1024, 2048, 7, 128, torch.bfloat16, seed=5)
    run_and_check(b, norm=True)
    assert np.isfinite(b["state"].float().cpu().numpy()).all()


def test_decode_out_of_range_slot_is_skipped_and_reported():
    """A slot index >= the number of slots in a decode batch: the decode kernel
    reads and writes no slot for that request (zero history) and raises the
    error flag, which packed_dynamic_conv_checked reports as IndexError."""
    from greta_plugin_b200.vllm_conv import packed_dynamic_conv_checked

    b = make_batch([1, 1, 1, 1], [2, 99, 0, -1], [1, 1, 1, 1], 4, 256, 4, 1, torch.bfloat16, seed=31)
    st = b["state"].clone()
    with pytest.raises(IndexError):
        packed_dynamic_conv_checked(b["x"].to(DEV), b["w"].to(DEV), b["gate"].to(DEV), b["state"],
                                    b["starts"].to(DEV), b["slots"].to(DEV), b["init"].to(DEV), 1)
    # slots 1 and 3 are named by no valid request: untouched
    for s in (1, 3):
        assert torch.equal(st[s], b["state"][s])
