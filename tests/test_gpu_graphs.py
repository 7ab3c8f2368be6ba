"""CUDA-graph capture of the SSA path (tensor-core kernels, through the public API).

The drop-in contract asks for a path a training loop can capture: no host reads, no host
synchronisation, workspace and outputs from the caching allocator, kernels on the caller's
stream, launch attributes set once per device before capture. These tests capture forward and
backward of the autograd Function, replay the graph on new input values and compare with eager
calls on the same values; and graph the Megatron-style module with
torch.cuda.make_graphed_callables. Tolerance: replay and eager run the same kernels, so
everything but dq (fp32 L2 reduce-adds in unfixed order) must match exactly; dq within one
bf16 ulp.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _close(name, a, b):
    if name == "dq":
        d = (a.float() - b.float()).abs()
        assert (d <= b.float().abs() * 2 ** -7 + 1e-6).all(), name
    else:
        assert torch.equal(a, b), name


def test_capture_forward_backward_and_replay(cuda_device):
    from SSA.ssa_flash_attention import ssa_flash_attention
    dev = cuda_device
    B, Hq, Hkv, N, D = 2, 8, 2, 512, 64
    g = torch.Generator(device="cpu").manual_seed(7)

    def sample():
        q = (torch.randn(B, Hq, N, D, generator=g) * 0.5).to(torch.bfloat16)
        k = (torch.randn(B, Hkv, N, D, generator=g) * 0.5).to(torch.bfloat16)
        v = (torch.randn(B, Hkv, N, D, generator=g) * 0.5).to(torch.bfloat16)
        do = torch.randn(B, Hq, N, D, generator=g).to(torch.bfloat16)
        return [t.to(dev) for t in (q, k, v, do)]

    n = torch.full((Hq,), 0.6, device=dev, requires_grad=True)
    b = torch.tensor(0.8, device=dev)
    static = [t.clone() for t in sample()]
    sq, sk, sv = (t.requires_grad_(True) for t in static[:3])
    sdo = static[3]

    def fwd_bwd():
        for t in (sq, sk, sv, n):
            t.grad = None
        out = ssa_flash_attention(sq, sk, sv, D ** -0.5, n, b, True)
        out.backward(sdo)
        return out

    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):  # warm-up on a side stream, as capture requires
        for _ in range(2):
            fwd_bwd()
    torch.cuda.current_stream(dev).wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    for t in (sq, sk, sv, n):
        t.grad = None
    with torch.cuda.graph(graph):
        static_out = ssa_flash_attention(sq, sk, sv, D ** -0.5, n, b, True)
        static_out.backward(sdo)
    grads = (sq.grad, sk.grad, sv.grad, n.grad)

    for _ in range(2):
        new = sample()
        with torch.no_grad():
            for dst, src in zip((sq, sk, sv, sdo), new):
                dst.copy_(src)
        graph.replay()
        torch.cuda.synchronize(dev)
        qe, ke, ve = (t.detach().clone().requires_grad_(True) for t in new[:3])
        ne = n.detach().clone().requires_grad_(True)
        oe = ssa_flash_attention(qe, ke, ve, D ** -0.5, ne, b, True)
        oe.backward(new[3])
        torch.cuda.synchronize(dev)
        _close("out", static_out, oe.detach())
        for name, a, e in zip(("dq", "dk", "dv", "dn"), grads, (qe.grad, ke.grad, ve.grad, ne.grad)):
            _close(name, a, e)
    del graph


def test_make_graphed_callables_module(cuda_device):
    from SSA.ssa_triton_attention import SSAAttentionConfig, SSATritonAttention
    dev = cuda_device
    S, B, Hq, Hkv, D = 256, 2, 8, 2, 64
    cfg = SSAAttentionConfig(num_attention_heads=Hq, kv_channels=D, num_query_groups=Hkv)
    mod = SSATritonAttention(cfg, layer_number=1, ssa_n=1.2, ssa_b=0.8).to(dev)
    g = torch.Generator(device="cpu").manual_seed(11)

    def sample():
        return [(torch.randn(S, B, h, D, generator=g) * 0.5).to(torch.bfloat16).to(dev)
                .requires_grad_(True) for h in (Hq, Hkv, Hkv)]

    class Core(torch.nn.Module):  # make_graphed_callables wants tensor-only positional args
        def __init__(self, m):
            super().__init__()
            self.m = m

        def forward(self, q, k, v):
            return self.m(q, k, v, None)

    core = Core(mod)
    graphed = torch.cuda.make_graphed_callables(core, tuple(sample()))
    q, k, v = sample()
    grad = torch.randn(S, B, Hq * D, generator=g).to(torch.bfloat16).to(dev)
    out = graphed(q, k, v)
    out.backward(grad)
    qe, ke, ve = (t.detach().clone().requires_grad_(True) for t in (q, k, v))
    n_grad_graph = mod.ssa_n_raw.grad.clone()
    mod.ssa_n_raw.grad = None
    oe = core(qe, ke, ve)
    oe.backward(grad)
    torch.cuda.synchronize(dev)
    _close("out", out.detach(), oe.detach())
    _close("dq", q.grad, qe.grad)
    _close("dk", k.grad, ke.grad)
    _close("dv", v.grad, ve.grad)
    _close("dn", n_grad_graph, mod.ssa_n_raw.grad)


def test_capture_with_fused_dropout(cuda_device):
    """Output dropout under capture: the seed is drawn inside the graph from torch's CUDA
    generator, so every replay draws a fresh mask, and each replay's output is the undropped
    output masked by the oracle's Philox mask for the seed that replay drew."""
    from oracle.ssa_dropout import keep_mask_dense, keep_scale, seed_pair
    from SSA.ssa_flash_attention import ssa_flash_attention
    from SSA.ssa_triton_kernel import make_dropout_seed
    dev = cuda_device
    B, Hq, Hkv, N, D, p = 1, 4, 2, 256, 64, 0.3
    g = torch.Generator(device="cpu").manual_seed(11)
    q, k, v = ((torch.randn(B, h, N, D, generator=g) * 0.5).to(torch.bfloat16).to(dev)
               for h in (Hq, Hkv, Hkv))
    n, b = torch.tensor(0.5, device=dev), torch.tensor(0.8, device=dev)
    seed_out = torch.zeros(2, dtype=torch.int64, device=dev)

    def step():
        seed = make_dropout_seed(dev)
        seed_out.copy_(seed)
        return ssa_flash_attention(q, k, v, D ** -0.5, n, b, True, dropout_p=p, training=True,
                                   dropout_seed=seed)

    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        step()
    torch.cuda.current_stream(dev).wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = step()
    plain = ssa_flash_attention(q, k, v, D ** -0.5, n, b, True).double().cpu()
    masks = []
    for _ in range(2):
        graph.replay()
        torch.cuda.synchronize()
        s0, s1 = seed_pair(seed_out)
        keep = torch.from_numpy(keep_mask_dense(B, Hq, N, D, s0, s1, p))
        got = out.double().cpu()
        assert (got[~keep] == 0).all()
        want = plain * keep_scale(p)
        kept = keep & (plain != 0)
        assert ((got - want).abs()[kept] <= 2.0 ** -6 * want.abs()[kept]).all()
        masks.append(keep)
    assert not torch.equal(masks[0], masks[1]), "replays must draw fresh masks"
    del graph
