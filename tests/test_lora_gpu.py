"""Parity of the adapted linear (quantized base + LoRA branch) with the oracle.

The oracle computes the reference graph (lib/torobi/dsl/layers.rb:16-25,
lib/torobi/lora.rb:79-85) in bf16 with every op rounded, and its VJP.
Tolerance: max rel err 1e-2 for y, dx, dA and dB.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from _util import dev_bf16, dev_u32, host_bf16

TOL = 1e-2


def _run_adapted(tq, cuda, x, c, s, b, a, bl, scale, bits, group, bias=None, dy=None):
    import torch

    X = dev_bf16(x, cuda)
    A = dev_bf16(a, cuda)
    B = dev_bf16(bl, cuda)
    C, S, Bi = dev_u32(c, cuda), dev_bf16(s, cuda), dev_bf16(b, cuda)
    ts, ts_t = tq.lora_down(X, A, scale)
    y = tq.qlora_matmul(X, C, S, Bi, True, group, bits,
                        bias=dev_bf16(bias, cuda) if bias is not None else None,
                        lora_up=B, lora_down=ts)
    out = {"y": y.float().cpu().numpy()}
    if dy is not None:
        DY = dev_bf16(dy, cuda)
        bt = tq.transpose_to_bf16(B.float())
        us, us_t = tq.lora_down(DY, bt, scale)
        dx = tq.qlora_matmul(DY, C, S, Bi, False, group, bits, lora_up=A, lora_down=us)
        db = tq.lora_grad(DY, ts_t, 0)
        da = tq.lora_grad(X, us_t, 1)
        torch.cuda.synchronize()
        out.update(dx=dx.float().cpu().numpy(), da=da.cpu().numpy(), db=db.cpu().numpy())
    return out


CASES = [
    # (m, n, k, rank, alpha, bits, group, with_bias)
    (512, 4864, 896, 8, 16.0, 4, 64, False),   # the single QLoRA linear workload
    (48, 136, 192, 8, 16.0, 4, 64, True),
    (200, 264, 384, 16, 32.0, 4, 32, False),
    (130, 512, 256, 16, 32.0, 8, 128, True),
    (64, 128, 128, 8, 8.0, 8, 64, False),
    # scale tiles staged by TMA (groups per row a multiple of 8)
    (300, 520, 1024, 16, 32.0, 4, 64, True),
    (96, 1024, 2048, 8, 16.0, 8, 32, False),
    # small m: split-K (LoRA added by the first split only, bias by the reduce)
    (32, 1024, 2048, 16, 32.0, 4, 64, True),
    # large: CTA pairs, token tile 128 then 256 both ways
    (1536, 3072, 2560, 16, 32.0, 4, 64, True),
    (2304, 4096, 2560, 8, 16.0, 8, 32, False),
]


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES, ids=lambda c: "m{}_n{}_k{}_r{}".format(*c[:4]))
def test_adapted_linear_forward_and_backward(cuda, oracle, case):
    import torobi_b200 as tq

    m, n, k, r, alpha, bits, group, with_bias = case
    rng = np.random.default_rng(1)
    x = oracle.normal_bf16(rng, (m, k))
    w = oracle.normal_bf16(rng, (n, k), 0.02)
    a = oracle.normal_bf16(rng, (r, k), 1.0 / 8.0)
    bl = oracle.normal_bf16(rng, (n, r), 0.01)
    bias = oracle.normal_bf16(rng, (n,), 0.1) if with_bias else None
    dy = oracle.normal_bf16(rng, (m, n))
    c, s, b = oracle.quantize(w, bits, group)
    scale = alpha / r
    f = oracle.f32_from_bf16
    y_ref, _ = oracle.qlora_linear_fwd(f(x), c, s, b, f(a), f(bl), scale, bits, group,
                                       bias=f(bias) if bias is not None else None)
    dx_ref, da_ref, db_ref = oracle.qlora_linear_bwd(f(x), f(dy), c, s, b, f(a), f(bl), scale,
                                                     bits, group)
    got = _run_adapted(tq, cuda, x, c, s, b, a, bl, scale, bits, group, bias, dy)
    for name, ref in (("y", y_ref), ("dx", dx_ref), ("da", da_ref), ("db", db_ref)):
        err = oracle.rel_err(got[name], ref)
        assert err <= TOL, f"{name}: max rel err {err:.3e}"


@pytest.mark.gpu
def test_golden_qlora_fixture(cuda, oracle):
    import torobi_b200 as tq

    g = np.load(Path(__file__).parent / "golden" / "qlora.npz")
    M, K, N, r, alpha, bits, group = (int(v) for v in g["meta"])
    got = _run_adapted(tq, cuda, g["x"], g["codes"], g["scales"], g["biases"], g["lora_a"],
                       g["lora_b"], alpha / r, bits, group, g["bias"], g["dy"])
    f = oracle.f32_from_bf16
    for name in ("y", "dx", "da", "db"):
        err = oracle.rel_err(got[name], f(g[name]))
        assert err <= TOL, f"{name}: max rel err {err:.3e}"


@pytest.mark.gpu
def test_zero_lora_b_gives_the_base_model_exactly(cuda, oracle):
    """B starts at zero, so the adapted linear equals the base linear exactly
    (the reference's test/lora_test.rb:140-148 asks the same of logits)."""
    import torobi_b200 as tq

    rng = np.random.default_rng(3)
    m, n, k, r = 300, 384, 512, 16
    x = oracle.normal_bf16(rng, (m, k))
    w = oracle.normal_bf16(rng, (n, k), 0.02)
    a = oracle.normal_bf16(rng, (r, k), 0.125)
    bl = np.zeros((n, r), np.uint16)
    c, s, b = oracle.quantize(w, 4, 64)
    X = dev_bf16(x, cuda)
    C, S, Bi = dev_u32(c, cuda), dev_bf16(s, cuda), dev_bf16(b, cuda)
    base = tq.quantized_matmul(X, C, S, Bi, True, 64, 4)
    ts, _ = tq.lora_down(X, dev_bf16(a, cuda), 2.0)
    adapted = tq.qlora_matmul(X, C, S, Bi, True, 64, 4, lora_up=dev_bf16(bl, cuda), lora_down=ts)
    assert np.array_equal(base.float().cpu().numpy(), adapted.float().cpu().numpy())


@pytest.mark.gpu
def test_lora_grad_accumulates_micro_batches(cuda, oracle):
    """Gradients of two halves accumulated equal the gradient of the whole
    (engine/src/state.rs:418-449: the gradient of a sum is the sum)."""
    import torch
    import torobi_b200 as tq

    torch.manual_seed(5)
    x = torch.randn(512, 640, device=cuda).bfloat16()
    p_t = torch.randn(16, 512, device=cuda).bfloat16()
    whole = tq.lora_grad(x, p_t.contiguous(), 1)
    acc = torch.zeros(16, 640, device=cuda)
    tq.lora_grad(x[:256], p_t[:, :256].contiguous(), 1, out=acc, accumulate=True)
    tq.lora_grad(x[256:], p_t[:, 256:].contiguous(), 1, out=acc, accumulate=True)
    # A ragged row count: the transposed operand carries a padded pitch.
    ragged = tq.lora_grad(x[:203], torch.nn.functional.pad(p_t[:, :203], (0, 5)).contiguous(), 1)
    assert torch.allclose(ragged, p_t[:, :203].float() @ x[:203].float(), rtol=1e-4, atol=1e-3)
    ref = (p_t.float() @ x.float())
    assert torch.allclose(whole, ref, rtol=1e-4, atol=1e-3)
    assert torch.allclose(acc, ref, rtol=1e-4, atol=1e-3)


@pytest.mark.gpu
@pytest.mark.parametrize("m,k,r", [(8192, 4096, 16),   # q/k/v/o/gate/up: k split in two
                                   (2048, 14336, 8),   # down_proj: four CTAs per row tile
                                   (4096, 896, 16),    # 14 k steps over four CTAs
                                   (300, 320, 16),     # 5 k steps over three, ragged rows
                                   (128, 64, 8)])      # one k step: no split
def test_lora_down_with_k_split_over_a_cluster(cuda, oracle, m, k, r):
    """The down-projection RNE(scale * x.A^T) when k is split over a cluster
    of CTAs (partials added in the leader's shared memory) against an f32
    reference, and its transposed copy bit-equal to it.  Then the adapter
    gradient x^T.P over the same x, one wave of CTAs each reducing a slice
    of m (one slice per tile at k = 14336)."""
    import torch
    import torobi_b200 as tq

    torch.manual_seed(11)
    x = torch.randn(m, k, device=cuda).bfloat16()
    a = (torch.randn(r, k, device=cuda) / 8).bfloat16()
    out, out_t = tq.lora_down(x, a, 2.0)
    want = (2.0 * (x.float() @ a.float().t())).cpu().numpy()
    err = oracle.rel_err(out.float().cpu().numpy(), want)
    assert err <= TOL, f"max rel err {err:.3e}"
    assert torch.equal(out_t[:, :m], out.t())
    again, _ = tq.lora_down(x, a, 2.0)
    assert torch.equal(again, out)  # the cluster reduction is deterministic
    g = tq.lora_grad(x, out_t, 0)
    g_ref = (x.float().t() @ out_t[:, :m].float().t()).cpu().numpy()
    err = oracle.rel_err(g.cpu().numpy(), g_ref)
    assert err <= 1e-4, f"grad: max rel err {err:.3e}"


@pytest.mark.gpu
@pytest.mark.parametrize("m,k,r", [(8192, 4096, 48),   # q/k/v stacked, r16 each
                                   (8192, 4096, 32),   # gate/up stacked
                                   (4096, 896, 16),    # Qwen q/v, r8 each
                                   (300, 320, 24),     # three r8 adapters, ragged rows
                                   (520, 1024, 64)])   # the widest stack
def test_stacked_down_projection_and_gradient(cuda, oracle, m, k, r):
    """Several adapters' A matrices stacked along the rank (linears that read
    one x): the down-projection of all of them in one pass equals the f32
    reference, each member's columns bit-equal to its own single-adapter
    launch; the stacked gradient P^T.x equals the f32 product."""
    import torch
    import torobi_b200 as tq

    torch.manual_seed(13)
    x = torch.randn(m, k, device=cuda).bfloat16()
    a = (torch.randn(r, k, device=cuda) / 8).bfloat16()
    out, out_t = tq.lora_down(x, a, 2.0)
    want = (2.0 * (x.float() @ a.float().t())).cpu().numpy()
    assert oracle.rel_err(out.float().cpu().numpy(), want) <= TOL
    assert torch.equal(out_t[:, :m], out.t())
    width = 8 if r % 16 else 16
    for c0 in range(0, r, width):
        one, _ = tq.lora_down(x, a[c0:c0 + width].contiguous(), 2.0)
        assert torch.equal(one, out[:, c0:c0 + width]), c0
    g = tq.lora_grad(x, out_t, 1)
    g_ref = (out_t[:, :m].float() @ x.float()).cpu().numpy()
    assert oracle.rel_err(g.cpu().numpy(), g_ref) <= 1e-4
    # The backward writes each member's transposed rows into its slice.
    buf = torch.zeros(r, out_t.shape[1], dtype=torch.bfloat16, device=cuda)
    for c0 in range(0, r, width):
        tq.lora_down(x, a[c0:c0 + width].contiguous(), 2.0, out_t=buf[c0:c0 + width])
    assert torch.equal(buf[:, :m], out_t[:, :m])


@pytest.mark.gpu
def test_gemm_reads_an_adapter_s_columns_of_a_stacked_down_projection(cuda):
    """qlora_matmul given a column slice of a stacked [m, R] down-projection
    (row pitch R) equals the call on a contiguous copy of those columns, bit
    for bit, on the single-CTA, split-K and pair paths."""
    import torch
    import torobi_b200 as tq

    torch.manual_seed(17)
    for m, n, k in ((300, 1032, 1024), (32, 1024, 2048), (1536, 3072, 2560)):
        w = (torch.randn(n, k, device=cuda) * 0.02).bfloat16()
        c, s, b = tq.quantize(w, 64, 4)
        x = torch.randn(m, k, device=cuda).bfloat16()
        stack = torch.randn(m, 48, device=cuda).bfloat16()
        up = (torch.randn(n, 16, device=cuda) * 0.05).bfloat16()
        for c0 in (0, 16, 32):
            got = tq.qlora_matmul(x, c, s, b, True, 64, 4, lora_up=up,
                                  lora_down=stack[:, c0:c0 + 16])
            want = tq.qlora_matmul(x, c, s, b, True, 64, 4, lora_up=up,
                                   lora_down=stack[:, c0:c0 + 16].contiguous())
            assert torch.equal(got, want), (m, n, k, c0)


@pytest.mark.gpu
@pytest.mark.parametrize("targets", [("q_proj", "k_proj", "v_proj"), ("q_proj", "v_proj")])
def test_grouped_linears_match_one_linear_at_a_time(cuda, targets):
    """qlora_linears over q/k/v (one stacked down-projection and one dA pass)
    gives the outputs of three qlora_linear calls bit for bit, and the same
    input gradient and adapter gradients to summation order."""
    import torch

    from torobi_b200.qlora import LoRAStore, QuantizedWeight, qlora_linear, qlora_linears

    torch.manual_seed(19)
    d_in, outs = 512, {"q_proj": 512, "k_proj": 128, "v_proj": 128}
    ws = [QuantizedWeight.from_dense((torch.randn(o, d_in, device=cuda) * 0.02).bfloat16(),
                                     4, 64, torch.randn(o, device=cuda).bfloat16())
          for o in outs.values()]
    stores = []
    for grouped in (True, False):
        st = LoRAStore(cuda)
        for name, o in outs.items():
            if name in targets:
                st.declare(name, d_in, o, 16, 32.0, group="qkv" if grouped else None)
        st.materialize(torch.Generator(device=cuda).manual_seed(3))
        for ad in st.adapters.values():
            ad.b.normal_(0.0, 0.05, generator=torch.Generator(device=cuda).manual_seed(4))
        st.refresh_bf16(full=True)
        stores.append(st)
    x = torch.randn(2, 96, d_in, device=cuda).bfloat16()
    dys = [torch.randn(2, 96, o, device=cuda).bfloat16() for o in outs.values()]
    res = []
    for st, grouped in zip(stores, (True, False)):
        ads = [st.adapters.get(n) for n in outs]
        xi = x.clone().requires_grad_()
        ys = qlora_linears(xi, ws, ads) if grouped else [qlora_linear(xi, w, ad)
                                                          for w, ad in zip(ws, ads)]
        torch.autograd.backward(ys, dys)
        res.append((ys, xi.grad, st.grads.clone()))
    (y1, dx1, g1), (y2, dx2, g2) = res
    assert len(stores[0].groups) == 1 and not stores[1].groups
    for a, b in zip(y1, y2):
        assert torch.equal(a, b)
    assert ((dx1.float() - dx2.float()).abs().max() / dx2.float().abs().max()).item() < 1e-2
    assert ((g1 - g2).abs().max() / g2.abs().max()).item() < 1e-4
