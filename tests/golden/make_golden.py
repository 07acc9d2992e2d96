"""Generate the golden vectors under tests/golden/ by running the REFERENCE.

Run in a checkout that has the reference (Garbo-AI/greta-plugin) on disk:

    python tests/golden/make_golden.py --reference /path/to/greta-plugin

The reference's own code computes every expected output here:
  * its pure-torch paths (torch_dynamic_causal_conv1d with autograd,
    greta_vllm.conv.packed_dynamic_conv, the HF torch decode/from-context), and
  * its Triton kernels executed by the Triton CPU interpreter
    (TRITON_INTERPRET=1): dynconv_fwd/bwd/inference/decode kernels and
    packed_dynamic_conv_triton (_conv_kernel + _state_kernel).
Autotuned kernels are called through `.fn.fn[grid]` with an explicit BD,
because the autotuner needs a GPU benchmarker.

Outputs: one compressed .npz per case (inputs + expected outputs, fp32 or the
raw uint16 bits of bf16 tensors) and config1_stats.json (config 1 is too large
to store: its inputs are regenerated from the seed, and the fixture holds
checksums of inputs and outputs plus sampled output entries).
"""
from __future__ import annotations

import argparse
import json
import os
import sys
from pathlib import Path

OUT = Path(__file__).resolve().parent


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("GRETA_REFERENCE"),
                    help="checkout of Garbo-AI/greta-plugin (or set GRETA_REFERENCE)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("pass --reference <checkout of the reference> or set GRETA_REFERENCE")
    os.environ["TRITON_INTERPRET"] = "1"
    sys.path.insert(0, args.reference)

    import numpy as np
    import torch
    import triton

    import greta.dynamic_conv as dc
    import greta.modeling_greta as mg
    import greta_vllm.conv as vconv
    import greta_vllm.triton_conv as vtc

    torch.manual_seed(0)

    def bits(t):
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)

    def f32(t):
        return t.detach().float().contiguous().numpy()

    def save(name, **arrays):
        np.savez_compressed(OUT / f"{name}.npz", **arrays)
        print("wrote", name, {k: getattr(v, "shape", v) for k, v in arrays.items()})

    def gen(seed):
        return torch.Generator().manual_seed(seed)

    # ------------------------------------------------------------------
    # training forward / backward (fp32): torch reference + interpreter
    # ------------------------------------------------------------------
    def train_case(name, seed, cu, D, W, G, norm, gate_on, bd):
        g = gen(seed)
        T = cu[-1]
        x = torch.randn(1, T, D, generator=g)
        w = torch.randn(T, W, D // G, generator=g) * (1.0 / W) ** 0.5
        gate = torch.randn(1, T, D, generator=g) if gate_on else None
        dout = torch.randn(1, T, D, generator=g)
        cu_t = torch.tensor(cu, dtype=torch.int32)
        eps = 1e-6
        xr, wr = x.clone().requires_grad_(), w.clone().requires_grad_()
        gr = gate.clone().requires_grad_() if gate_on else None
        y = dc.torch_dynamic_causal_conv1d(xr, wr, gr, cu_t, G, norm, eps)
        y.backward(dout)
        out = dict(x=f32(x[0]), w=f32(w), dout=f32(dout[0]), cu_seqlens=np.array(cu, np.int64),
                   D=D, W=W, G=G, norm=int(norm), eps=eps,
                   y_torch=f32(y[0]), dx_torch=f32(xr.grad[0]), dw_torch=f32(wr.grad))
        if gate_on:
            out.update(gate=f32(gate[0]), dg_torch=f32(gr.grad[0]))
        # the reference Triton kernels, interpreted
        BT = 16
        ci = dc.prepare_chunk_indices(cu_t, BT)
        NT = len(ci)
        yk = torch.empty_like(x)
        yr = torch.empty_like(x) if norm else None
        dc.dynconv_fwd_kernel.fn.fn[(NT, triton.cdiv(D, bd), 1)](
            x=x, w=w, g=gate, y=yk, yr=yr, cu_seqlens=cu_t, chunk_indices=ci, T=T, eps=eps, D=D, G=G, W=W,
            BT=BT, HAS_NORM=norm, IS_VARLEN=True, HAS_GATE=gate_on, SAVE_PRE=yr is not None, BD=bd)
        dx = torch.empty_like(x)
        dw = torch.empty_like(w)
        dg = torch.empty_like(gate) if gate_on else None
        dc.dynconv_bwd_kernel.fn.fn[(NT, triton.cdiv(D, bd), 1)](
            x=x, w=w, g=gate, yr=yr, dout=dout, dx=dx, dw=dw, dg=dg, cu_seqlens=cu_t, chunk_indices=ci, T=T,
            eps=eps, D=D, G=G, W=W, BT=BT, HAS_NORM=norm, IS_VARLEN=True, HAS_GATE=gate_on, BD=bd)
        out.update(y_triton=f32(yk[0]), dx_triton=f32(dx[0]), dw_triton=f32(dw))
        if norm:
            out.update(yr_triton=f32(yr[0]))
        if gate_on:
            out.update(dg_triton=f32(dg[0]))
        save(name, **out)

    # ragged lengths include 1 and 2 (< W-1) so history masking is exercised
    train_case("train_g1_w4_plain", 1, [0, 1, 3, 20, 21, 45], 64, 4, 1, False, False, 16)
    train_case("train_g4_w4_norm_gate", 2, [0, 2, 19, 40], 64, 4, 4, True, True, 16)
    train_case("train_g16_w7_norm_gate", 3, [0, 5, 6, 30], 64, 7, 16, True, True, 32)
    train_case("train_g128_w7_norm_gate", 4, [0, 3, 24], 256, 7, 128, True, True, 128)
    train_case("train_g2_w3_gate", 5, [0, 17, 18, 33], 32, 3, 2, False, True, 16)

    # ------------------------------------------------------------------
    # training forward, bf16 through the interpreted kernel
    # ------------------------------------------------------------------
    g = gen(6)
    T, D, W, G = 37, 64, 4, 8
    cu = [0, 2, 15, 37]
    x = torch.randn(1, T, D, generator=g).bfloat16()
    w = (torch.randn(T, W, D // G, generator=g) * 0.5).bfloat16()
    gate = torch.randn(1, T, D, generator=g).bfloat16()
    cu_t = torch.tensor(cu, dtype=torch.int32)
    ci = dc.prepare_chunk_indices(cu_t, 16)
    y = torch.empty_like(x)
    yr = torch.empty_like(x)
    dc.dynconv_fwd_kernel.fn.fn[(len(ci), D // 16, 1)](
        x=x, w=w, g=gate, y=y, yr=yr, cu_seqlens=cu_t, chunk_indices=ci, T=T, eps=1e-6, D=D, G=G, W=W, BT=16,
        HAS_NORM=True, IS_VARLEN=True, HAS_GATE=True, SAVE_PRE=True, BD=16)
    save("train_bf16_g8_w4_norm_gate", x_bits=bits(x[0]), w_bits=bits(w), gate_bits=bits(gate[0]),
         cu_seqlens=np.array(cu, np.int64), D=D, W=W, G=G, norm=1, eps=1e-6,
         y_bits=bits(y[0]), yr_bits=bits(yr[0]))

    # ------------------------------------------------------------------
    # HF inference from context (interpreted kernel) + torch from_context
    # ------------------------------------------------------------------
    g = gen(7)
    B, Q, D, W, G = 2, 5, 64, 4, 8
    ctx = torch.randn(B, Q + W - 1, D, generator=g)
    w = torch.randn(B, Q, W, D // G, generator=g) * 0.5
    gate = torch.randn(B, Q, D, generator=g)
    y = torch.empty(B, Q, D)
    dc.dynconv_inference_kernel.fn.fn[(triton.cdiv(Q, 16), D // 16, B)](
        context=ctx, w=w, g=gate, y=y, Q=Q, eps=1e-6, D=D, G=G, W=W, BT=16, HAS_NORM=True, HAS_GATE=True, BD=16)
    y_torch = mg.torch_dynamic_causal_conv1d_from_context(ctx, w, gate, G, True, 1e-6)
    save("inference_g8_w4_norm_gate", context=f32(ctx), w=f32(w), gate=f32(gate), D=D, W=W, G=G, norm=1,
         eps=1e-6, y_triton=f32(y), y_torch=f32(y_torch))

    # ------------------------------------------------------------------
    # HF decode by batch row (interpreted kernel); state shifted in place
    # ------------------------------------------------------------------
    for name, seed, W, G, norm in [("decode_rows_g4_w4_norm_gate", 8, 4, 4, True),
                                   ("decode_rows_g1_w2_gate", 9, 2, 1, False)]:
        g = gen(seed)
        B, D = 3, 64
        x = torch.randn(B, D, generator=g)
        w = torch.randn(B, W, D // G, generator=g) * 0.5
        gate = torch.randn(B, D, generator=g)
        state = torch.randn(B, D, W - 1, generator=g)
        st = state.clone()
        y = torch.empty(B, D)
        dc.dynconv_decode_kernel[(triton.cdiv(D, 128), B)](
            x=x, w=w, g=gate, conv_state=st, y=y, eps=1e-6, D=D, G=G, W=W, BD=128, HAS_NORM=norm)
        st_t = state.clone()
        y_torch = mg.torch_dynamic_causal_conv1d_decode(x, w, gate, st_t, G, norm, 1e-6)
        save(name, x=f32(x), w=f32(w), gate=f32(gate), state=f32(state), D=D, W=W, G=G, norm=int(norm), eps=1e-6,
             y_triton=f32(y), state_triton=f32(st), y_torch=f32(y_torch), state_torch=f32(st_t))

    # ------------------------------------------------------------------
    # vLLM packed batch: interpreted _conv_kernel + _state_kernel (handles
    # slot -1) and the torch packed_dynamic_conv on the non-padding requests.
    # ------------------------------------------------------------------
    def packed_case(name, seed, lengths, slots, init, n_slots, D, W, G, norm, gate_on, sd_layout, dtype):
        g = gen(seed)
        T = sum(lengths)
        starts = torch.tensor([0] + list(np.cumsum(lengths)), dtype=torch.int32)
        x = torch.randn(T, D, generator=g).to(dtype)
        w = (torch.randn(T, W, D // G, generator=g) * 0.5).to(dtype)
        gate = torch.randn(T, D, generator=g).to(dtype) if gate_on else None
        base = torch.randn(n_slots, D, W - 1, generator=g).to(dtype)
        if sd_layout:
            storage = base.transpose(1, 2).contiguous()  # [slots, W-1, D] storage
            state = storage.transpose(1, 2)               # [slots, D, W-1] view, strides (.., 1, D)
        else:
            storage = base.clone()
            state = storage
        slots_t = torch.tensor(slots, dtype=torch.int32)
        init_t = torch.tensor(init, dtype=torch.int8)
        y = vtc.packed_dynamic_conv_triton(x, w, gate, state, starts, slots_t, init_t, G, norm=norm, eps=1e-6)
        out = dict(starts=starts.numpy().astype(np.int64), slots=np.array(slots, np.int64),
                   has_initial=np.array(init, np.int64), D=D, W=W, G=G, norm=2 if norm else 0, eps=1e-6,
                   sd_layout=int(sd_layout))
        if dtype == torch.float32:
            out.update(x=f32(x), w=f32(w), state=f32(base), y_triton=f32(y), state_triton=f32(state))
            if gate_on:
                out.update(gate=f32(gate))
            keep = [i for i, s in enumerate(slots) if s >= 0]
            if len(keep) == len(slots):
                st2 = base.clone()
                y2 = vconv.packed_dynamic_conv(x, w, gate, st2, starts, slots_t, init_t, G, norm=norm, eps=1e-6)
                out.update(y_torch=f32(y2), state_torch=f32(st2))
        else:
            out.update(x_bits=bits(x), w_bits=bits(w), state_bits=bits(base), y_bits=bits(y),
                       state_out_bits=bits(state.contiguous()))
            if gate_on:
                out.update(gate_bits=bits(gate))
        save(name, **out)

    # decodes first (length 1), then prefills; a slot of -1; has_initial mix;
    # a prefill shorter than W-1 that must shift old history.
    packed_case("packed_stable_gate_mixed", 10, [1, 1, 1, 2, 9, 16], [5, -1, 2, 7, 0, 3], [1, 1, 0, 1, 1, 0],
                8, 64, 4, 8, True, True, False, torch.float32)
    packed_case("packed_all_valid_torchcheck", 11, [1, 3, 12], [4, 1, 6], [1, 1, 0], 8, 64, 4, 4, True, True,
                False, torch.float32)
    packed_case("packed_sd_layout_w7_g16", 12, [1, 4, 20], [2, 0, 5], [1, 1, 1], 6, 64, 7, 16, True, True, True,
                torch.float32)
    packed_case("packed_nonorm_nogate_g1", 13, [2, 1, 7], [1, 3, -1], [1, 0, 1], 4, 32, 4, 1, False, False,
                False, torch.float32)
    packed_case("packed_bf16_stable_gate", 14, [1, 1, 2, 13], [3, 0, -1, 6], [1, 1, 1, 1], 8, 64, 4, 8, True,
                True, False, torch.bfloat16)

    # ------------------------------------------------------------------
    # config 1 (CPU-runnable correctness): fp32, 2 x 256 packed, C=512, K=4,
    # forward only, seed 0; too large to store -> checksums + samples.
    # ------------------------------------------------------------------
    g = gen(0)
    x = torch.randn(1, 512, 512, generator=g)
    w = torch.randn(512, 4, 512, generator=g) * 0.5
    cu_t = torch.tensor([0, 256, 512], dtype=torch.int32)
    y = dc.torch_dynamic_causal_conv1d(x, w, None, cu_t, 1, False)
    idx = torch.randint(0, 512 * 512, (512,), generator=gen(123))
    stats = dict(
        seed=0, shape_x=[1, 512, 512], shape_w=[512, 4, 512], w_scale=0.5, cu_seqlens=[0, 256, 512],
        x_sum=float(x.double().sum()), x_sq=float(x.double().square().sum()),
        w_sum=float(w.double().sum()), w_sq=float(w.double().square().sum()),
        y_sum=float(y.double().sum()), y_sq=float(y.double().square().sum()),
        y_abs=float(y.double().abs().sum()),
        sample_idx=idx.tolist(), sample_val=y.reshape(-1)[idx].tolist(),
    )
    (OUT / "config1_stats.json").write_text(json.dumps(stats))
    print("wrote config1_stats.json")


if __name__ == "__main__":
    main()
