"""The NF4 GEMM with the decode in the tensor-core kernel (tb_nf4_gemm) against the oracle
(bit-exact dequantisation, fp64 sums) and against cuBLAS over the unpacked weight, in both
directions."""

import numpy as np
import pytest
import torch

from helpers import assert_rel, nf4_weight
from oracle import nf4 as onf4
from oracle import ops

pytestmark = pytest.mark.gpu

# fp16 output of an fp32-accumulated sum: half an fp16 ulp of rounding plus the sum's order
RTOL = 1e-3


def _weights(rows, cols, nested, seed):
    rng = np.random.default_rng(seed)
    qs = [onf4.quantize((rng.standard_normal((r, cols)) * 0.05).astype(np.float16),
                        blocksize=64, nested=nested) for r in rows]
    return qs, [nf4_weight(q, "cuda") for q in qs]


def _x(rows, cols, seed, std=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(rows, cols, generator=g) * std).half().cuda()


@pytest.fixture(params=[0, 1], ids=["split", "no_split"])
def split_variant(request):
    """The reduction split over several work units (fp32 partials summed in split order) or
    never split; the automatic choice restored afterwards."""
    from testt_b200 import nf4_gemm

    nf4_gemm.set_variant(request.param)
    yield request.param
    nf4_gemm.set_variant(0)


@pytest.mark.parametrize("nested", [False, True])
@pytest.mark.parametrize("tokens", [1, 37, 621, 1000])
def test_forward_stacked_with_bias_matches_oracle(nested, tokens, split_variant):
    """q|k|v-shaped stack (the reduction split over several CTAs at these sizes), with bias."""
    from testt_b200 import nf4_gemm

    qs, ws = _weights((512, 128, 128), 1536, nested, seed=tokens)
    x = _x(tokens, 1536, seed=1)
    bias = _x(1, 768, seed=2, std=0.1)[0]
    out = nf4_gemm.nf4_matmul(x, ws, bias)
    torch.cuda.synchronize()
    assert_rel(out.cpu(), ops.nf4_matmul(x.cpu(), qs, bias.cpu()), RTOL, "forward")
    assert_rel(nf4_gemm.nf4_matmul(x, ws).cpu(), ops.nf4_matmul(x.cpu(), qs), RTOL, "no bias")


@pytest.mark.parametrize("nested", [False, True])
@pytest.mark.parametrize("tokens", [1, 300, 621])
def test_backward_stacked_matches_oracle(nested, tokens, split_variant):
    """dX = dY W over a stack of three weights (the reduction split over several CTAs, the
    splits' ranges crossing from one weight to the next)."""
    from testt_b200 import nf4_gemm

    qs, ws = _weights((640, 384, 512), 256, nested, seed=10 + tokens)
    dy = _x(tokens, 1536, seed=3, std=0.01)
    out = nf4_gemm.nf4_matmul(dy, ws, transpose=True)
    torch.cuda.synchronize()
    assert_rel(out.cpu(), ops.nf4_matmul(dy.cpu(), qs, transpose=True), RTOL, "backward")


@pytest.mark.parametrize("which", ["gate_up", "down"])
def test_config5_shapes_match_cublas_over_unpacked(which):
    """The step's MLP GEMMs at 621 tokens, both directions, against torch.matmul (cuBLAS) over
    tb_nf4_unpack's bit-exact fp16 weight."""
    from testt_b200 import _lib, nf4_gemm
    from testt_b200.nf4 import unpack_concat

    rows, cols = ((8960, 8960), 1536) if which == "gate_up" else ((1536,), 8960)
    _, ws = _weights(rows, cols, True, seed=7)
    w16 = unpack_concat(ws, "cuda")
    x = _x(621, cols, seed=4)
    dy = _x(621, sum(rows), seed=5, std=0.01)
    fwd = nf4_gemm.nf4_matmul(x, ws)
    bwd = nf4_gemm.nf4_matmul(dy, ws, transpose=True)
    ref_f = (x.float() @ w16.float().t()).half()
    ref_b = (dy.float() @ w16.float()).half()
    torch.cuda.synchronize()
    assert_rel(fwd.cpu(), ref_f.cpu(), RTOL, f"{which} forward")
    assert_rel(bwd.cpu(), ref_b.cpu(), RTOL, f"{which} backward")
    assert_rel(fwd.cpu(), torch.matmul(x, w16.t()).cpu(), RTOL, f"{which} vs cuBLAS")
    assert _lib.wait_timeouts() == 0


def test_rejects_shapes_it_does_not_take():
    from testt_b200 import nf4_gemm

    _, ws = _weights((64, 64), 256, False, seed=9)   # forward tiles of 128 rows would straddle
    with pytest.raises(ValueError):
        nf4_gemm.nf4_matmul(_x(4, 256, seed=6), ws)
    assert nf4_gemm.nf4_matmul(_x(0, 128, seed=6), ws, transpose=True).shape == (0, 256)


def test_fused_layer_nodes_match_the_unpacking_nodes():
    """fused_layer.layer_linear / layer_mlp (the GEMM decodes NF4 itself) against
    nf4.layer_linear / mlp.layer_mlp (one unpack launch, cuBLAS) on the same LayerWeights, forward
    and input gradient, at the Qwen2.5 layer's widths scaled down (q|k|v, o, gate|up, down)."""
    from testt_b200 import fused_layer, mlp, nf4

    rng = np.random.default_rng(12)
    shapes = [(512, 512), (128, 512), (128, 512), (512, 512), (1024, 512), (1024, 512), (512, 1024)]
    qs = [onf4.quantize((rng.standard_normal(sh) * 0.05).astype(np.float16), 64, nested=True)
          for sh in shapes]
    ws = [nf4_weight(q, "cuda") for q in qs]
    lw = nf4.LayerWeights(((ws[0], ws[1], ws[2]), (ws[3],), (ws[4], ws[5]), (ws[6],)))
    assert fused_layer.usable(lw)
    bias = _x(1, 768, seed=13, std=0.1)[0]
    x = _x(300, 512, seed=14).requires_grad_(True)
    x2 = x.detach().clone().requires_grad_(True)
    y = fused_layer.layer_linear(x, lw, 0, bias)
    z = fused_layer.layer_mlp(y[:, :512], lw, 2, 3)
    y2 = nf4.layer_linear(x2, lw, 0, bias)
    z2 = mlp.layer_mlp(y2[:, :512], lw, 2, 3)
    gz = _x(300, 512, seed=15, std=0.01)
    (z.float() * gz.float()).sum().backward()
    (z2.float() * gz.float()).sum().backward()
    lw.release()
    torch.cuda.synchronize()
    assert_rel(y.detach().cpu(), y2.detach().cpu(), 2e-3, "qkv")
    assert_rel(z.detach().cpu(), z2.detach().cpu(), 2e-3, "mlp")
    assert_rel(x.grad.cpu(), x2.grad.cpu(), 2e-3, "dx")


@pytest.mark.parametrize("tokens", [1, 300, 621])
def test_swiglu_epilogues_match_gemm_then_swiglu_kernels(tokens):
    """tb_nf4_gemm_swiglu: gate|up forward with act formed in the epilogue, and down's dX with
    the in-place SwiGLU backward in the epilogue, against the plain GEMM followed by the SwiGLU
    kernels (mlp.gated_silu / gated_silu_backward_)."""
    from testt_b200 import mlp, nf4_gemm

    inter, hidden = 1024, 512
    _, gate_up = _weights((inter, inter), hidden, True, seed=20)
    _, down = _weights((hidden,), inter, True, seed=21)
    x = _x(tokens, hidden, seed=22)
    gu, act = nf4_gemm.gate_up_swiglu(x, gate_up)
    gu_ref = nf4_gemm.nf4_matmul(x, gate_up)
    torch.cuda.synchronize()
    assert_rel(gu.cpu(), gu_ref.cpu(), RTOL, "gu")
    from helpers import assert_ulp

    assert_ulp(act.cpu(), mlp.gated_silu(gu).cpu(), 1, "act from the epilogue's own gu")
    dy = _x(tokens, hidden, seed=23, std=0.01)
    g1, g2 = gu.clone(), gu.clone()
    nf4_gemm.down_swiglu_backward_(dy, down[0], g1)
    dact = nf4_gemm.nf4_matmul(dy, down, transpose=True)
    mlp.gated_silu_backward_(dact, g2)
    torch.cuda.synchronize()
    assert_rel(g1.float().cpu(), g2.float().cpu(), 2e-3, "d(gate|up)")


@pytest.mark.parametrize("tokens", [1, 150, 621])
@pytest.mark.parametrize("lora", [True, False])
def test_qkv_rope_epilogue_matches_gemm_then_rope_tokens(tokens, lora):
    """tb_nf4_gemm_qkv_rope (bias, LoRA rows and the rotary embedding in the q|k|v GEMM's
    finishing phase, one head a tile, the split reduction through the cluster) against the
    plain GEMM followed by rope.rope_tokens."""
    from helpers import assert_ulp
    from oracle import ops
    from testt_b200 import nf4_gemm, rope

    nh, nkv, hidden, seq = 4, 2, 512, 512
    _, ws = _weights((nh * 128, nkv * 128, nkv * 128), hidden, True, seed=30)
    x = _x(tokens, hidden, seed=31)
    bias = _x(1, (nh + 2 * nkv) * 128, seed=32, std=0.1)[0]
    lq = _x(tokens, nh * 128, seed=33, std=0.01) if lora else None
    lv = _x(tokens, nkv * 128, seed=34, std=0.01) if lora else None
    cos, sin = (t.cuda() for t in ops.rope_tables(seq, 128, 1e6))
    g = torch.Generator().manual_seed(35)
    pos = torch.sort(torch.randperm(4 * seq, generator=g)[:tokens]).values.cuda()
    q, k, v = nf4_gemm.qkv_rope(x, ws, bias, lq, lv, cos, sin, pos, seq, nh, nkv)
    qkv = nf4_gemm.nf4_matmul(x, ws, bias)
    rq, rk, rv = rope.rope_tokens(qkv, lq, lv, cos, sin, pos, 4, seq, nh, nkv, 128)
    torch.cuda.synchronize()
    # the GEMM halves may round their fp32 sums differently (one fp16 ulp of qkv), then the
    # same arithmetic: held to the GEMM tolerance, and the v rows (no rotation) to one ulp
    assert_rel(q.float().cpu(), rq.float().cpu(), RTOL, "q")
    assert_rel(k.float().cpu(), rk.float().cpu(), RTOL, "k")
    assert_ulp(v.cpu(), rv.cpu(), 1, "v")


def test_fused_qkv_rope_node_matches_linear_then_rope_tokens():
    """fused_layer.qkv_rope (forward and the gradients of x and of both LoRA inputs) against
    nf4.layer_linear followed by rope.rope_tokens on the same LayerWeights."""
    from oracle import ops
    from testt_b200 import fused_layer, nf4, rope

    nh, nkv, hidden, seq, tokens = 4, 2, 512, 512, 300
    _, ws = _weights((nh * 128, nkv * 128, nkv * 128), hidden, True, seed=40)
    lw = nf4.LayerWeights((tuple(ws),))
    bias = _x(1, (nh + 2 * nkv) * 128, seed=41, std=0.1)[0]
    cos, sin = (t.cuda() for t in ops.rope_tables(seq, 128, 1e6))
    g = torch.Generator().manual_seed(42)
    pos = torch.sort(torch.randperm(4 * seq, generator=g)[:tokens]).values.cuda()
    ins = [_x(tokens, hidden, seed=43), _x(tokens, nh * 128, seed=44, std=0.01),
           _x(tokens, nkv * 128, seed=45, std=0.01)]
    a = [t.clone().requires_grad_(True) for t in ins]
    b = [t.clone().requires_grad_(True) for t in ins]
    out_a = fused_layer.qkv_rope(a[0], lw, 0, bias, a[1], a[2], cos, sin, pos, 4, seq, nh, nkv)
    qkv = nf4.layer_linear(b[0], lw, 0, bias, last=True)
    out_b = rope.rope_tokens(qkv, b[1], b[2], cos, sin, pos, 4, seq, nh, nkv, 128)
    grads = [_x(o.shape[0], o[0].numel(), seed=46 + i, std=0.01).view(o.shape)
             for i, o in enumerate(out_b)]
    torch.autograd.backward(out_a, grads)
    torch.autograd.backward(out_b, grads)
    lw.release()
    torch.cuda.synchronize()
    for x, y, name in zip(out_a, out_b, "qkv"):
        assert_rel(x.detach().float().cpu(), y.detach().float().cpu(), 2e-3, name)
    for x, y, name in zip(a, b, ("dx", "dlora_q", "dlora_v")):
        assert_rel(x.grad.float().cpu(), y.grad.float().cpu(), 2e-3, name)
