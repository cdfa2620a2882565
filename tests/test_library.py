"""The torch.library registration (``torch.ops.dsalt_b200.*``): shape functions on CPU
(fake tensors, no GPU), and on the GPU ``torch.compile(fullgraph=True)`` of the module —
which fails on any graph break — matching eager execution bit for bit, plus
``torch.library.opcheck`` of each operator (fake vs real outputs, schema)."""
import pytest
import torch

import dsalt_b200  # noqa: F401  (registers the operators)


def test_operators_registered_with_shape_functions():
    from torch._subclasses.fake_tensor import FakeTensorMode
    with FakeTensorMode():
        dev = "cuda"
        T, H, D, dm = 1100, 4, 64, 256
        q = torch.empty(T, H, D, dtype=torch.bfloat16, device=dev)
        x = torch.empty(T, dm, dtype=torch.bfloat16, device=dev)
        cu = torch.empty(3, dtype=torch.int32, device=dev)
        w, xn, vn = torch.ops.dsalt_b200.window_signals(x, x[0], x[0, :1], 16, 128, q, D, False, None)
        assert (w.shape, w.dtype, xn.shape, vn.shape) == ((T,), torch.int32, (T,), (T, H))
        lmk = torch.ops.dsalt_b200.select_landmarks(xn, vn, w, torch.empty(H, device=dev), cu, 32, H,
                                                    "block_causal", 512, [0, 600, 1100])
        assert lmk.shape == (H, 2 + 1, 32) and lmk.dtype == torch.int32
        g = torch.ops.dsalt_b200.select_landmarks(xn, vn, w, torch.empty(H, device=dev), cu, 32, H, "global", 512,
                                                  [0, 600, 1100])
        assert g.shape == (H, 2, 32)
        o = torch.ops.dsalt_b200.dsalt_attention(q, q, q, lmk, None, w, cu, 512, [0, 600, 1100], torch.float32)
        assert o.shape == q.shape and o.dtype == torch.float32
        c = torch.ops.dsalt_b200.core_forward(x, x[0], x[0, :1], 16, 128, torch.empty(H, device=dev), q, q, q, 32, cu,
                                              "global", 512, False, [0, 600, 1100], torch.bfloat16, None)
        assert c.shape == q.shape and c.dtype == torch.bfloat16


@pytest.mark.gpu
def test_compiled_module_fullgraph_matches_eager():
    from dsalt_b200 import DSALTAttention
    dev = torch.device("cuda", 0)
    torch.manual_seed(0)
    cu = [0, 700, 1900]
    mod = DSALTAttention(256, 4, 16, 256, 64, 2048, selection="block_causal", block=512).to(dev).eval()
    mod._collect_last_P = False  # the compiled graph covers the output path; _last_P is an eager metric
    x = torch.randn(cu[-1], 256, device=dev)
    cu_t = torch.tensor(cu, dtype=torch.int32, device=dev)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        ref, _ = mod(x, cu_t, cu_list=cu)
        torch._dynamo.reset()
        comp = torch.compile(mod, fullgraph=True, backend="aot_eager")
        got, _ = comp(x, cu_t, cu_list=cu)
    assert torch.equal(got, ref)


@pytest.mark.gpu
def test_opcheck_operators():
    from dsalt_b200 import ops
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(3)
    cu = [0, 600, 1100]
    T, H, D, dm = cu[-1], 4, 64, 256
    x = torch.randn(T, dm, device=dev, generator=g).bfloat16()
    q = torch.randn(T, H, D, device=dev, generator=g).bfloat16()
    k = torch.randn(T, H, D, device=dev, generator=g).bfloat16()
    v = torch.randn(T, H, D, device=dev, generator=g).bfloat16()
    gw = (torch.randn(dm, device=dev, generator=g) * 0.05).bfloat16()
    gb = torch.zeros(1, device=dev).bfloat16()
    alpha = torch.full((H,), 0.6, device=dev)
    cu_t = torch.tensor(cu, dtype=torch.int32, device=dev)
    w, xn, vn = ops.window_signals(x, gw, gb, 16, 256, v, D)
    lmk = ops.select_landmarks(xn, vn, w, alpha, cu_t, 32, H, "block_causal", 512, cu_list=cu)
    lib = torch.ops.dsalt_b200
    tests = ("test_schema", "test_faketensor")
    torch.library.opcheck(lib.window_signals, (x, gw, gb, 16, 256, v, D, False, None), test_utils=tests)
    torch.library.opcheck(lib.select_landmarks, (xn, vn, w, alpha, cu_t, 32, H, "block_causal", 512, cu),
                          test_utils=tests)
    torch.library.opcheck(lib.dsalt_attention, (q, k, v, lmk, None, w, cu_t, 512, cu, torch.bfloat16),
                          test_utils=tests)
    torch.library.opcheck(lib.core_forward, (x, gw, gb, 16, 256, alpha, q, k, v, 32, cu_t, "block_causal", 512,
                                             False, cu, torch.bfloat16, None), test_utils=tests)
