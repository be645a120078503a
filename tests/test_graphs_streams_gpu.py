"""Stream semantics of the C-ABI operators (reference contract
include/operatorlib/operators.h:8-46, docs/launcher_extraction.md:9-15:
enqueue-only, caller's stream, no global mutable state).

* CUDA-graph capture: every operator path is captured once and replayed
  after new data is copied into the captured input buffers; the replay must
  equal an eager call on the same data bit for bit (all kernels are
  deterministic, and stream-ordered workspaces become graph memory nodes).
* Concurrency: the same calls issued on two streams at once (independent
  buffers) must give exactly the sequential results, i.e. per-call
  workspaces are never shared.
"""
import numpy as np
import pytest

import operatorlib

pytestmark = pytest.mark.gpu


def _cases(torch, dev, rng):
    """(name, inputs, outputs, call(inputs, outputs)) for each operator path."""
    def t(a, dtype=None):
        x = torch.from_numpy(np.ascontiguousarray(a)).to(dev)
        return x.to(dtype) if dtype is not None else x

    f16 = torch.float16
    cases = []
    n = 3_000_017
    cases.append(("reduce", [t(rng.uniform(-1, 1, n).astype(np.float32))],
                  [torch.empty((), device=dev)],
                  lambda i, o: operatorlib.reduce_sum_into(i[0], o[0])))
    x = rng.normal(0, 2, (513, 1023)).astype(np.float32)
    cases.append(("softmax", [t(x)], [torch.empty(513, 1023, device=dev)],
                  lambda i, o: operatorlib.softmax_into(i[0], o[0])))
    x = rng.normal(0, 1, (300, 4096)).astype(np.float32)
    w = rng.normal(1, 0.1, 4096).astype(np.float32)
    cases.append(("rmsnorm", [t(x), t(w)], [torch.empty(300, 4096, device=dev)],
                  lambda i, o: operatorlib.rmsnorm_into(i[0], i[1], o[0], 1e-6)))
    x = rng.uniform(-1, 1, (777, 1029)).astype(np.float32)
    cases.append(("transpose", [t(x)], [torch.empty(1029, 777, device=dev)],
                  lambda i, o: operatorlib.transpose_into(i[0], o[0])))
    for name, (m, nn, k), dtype in [("gemm_pair", (512, 768, 512), f16),
                                    ("gemm_skinny", (7, 1024, 768), f16),
                                    ("gemm_ragged", (300, 517, 203), f16),
                                    ("gemm_f32_split", (2048, 2560, 256), None)]:
        a = (rng.uniform(-1, 1, (m, k)) / np.sqrt(k)).astype(np.float32)
        b = (rng.uniform(-1, 1, (k, nn)) / np.sqrt(k)).astype(np.float32)
        cases.append((name, [t(a, dtype), t(b, dtype)], [torch.empty(m, nn, device=dev)],
                      lambda i, o: operatorlib.gemm_into(i[0], i[1], o[0])))
    for name, shape, dtype, causal in [("attention_f16_split", (1, 3, 512, 128), f16, True),
                                       ("attention_f16_pairs", (2, 40, 1024, 64), f16, False),
                                       ("attention_f32_splitkv", (1, 2, 640, 128), None, False)]:
        q, k_, v = (rng.normal(0, 1, shape).astype(np.float32) for _ in range(3))
        cases.append((name, [t(q, dtype), t(k_, dtype), t(v, dtype)],
                      [torch.empty(shape, device=dev)],
                      lambda i, o, c=causal: operatorlib.attention_into(i[0], i[1], i[2], o[0], c)))
    return cases


def _fresh_like(torch, rng, x):
    y = torch.from_numpy(rng.standard_normal(tuple(x.shape)).astype(np.float32) * 0.5)
    return y.to(x.device).to(x.dtype)


@pytest.mark.parametrize("index", range(11))
def test_graph_capture_replay(cuda, index):
    import torch

    rng = np.random.default_rng(100 + index)
    name, ins, outs, call = _cases(torch, cuda, rng)[index]
    side = torch.cuda.Stream(cuda)
    side.wait_stream(torch.cuda.current_stream(cuda))
    with torch.cuda.stream(side):
        call(ins, outs)  # first call: one-time set-up outside the capture
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=side):
            call(ins, outs)
        for _ in range(2):
            new = [_fresh_like(torch, rng, x) for x in ins]
            for dst, src in zip(ins, new):
                dst.copy_(src)
            g.replay()
            got = [o.clone() for o in outs]
            eager = [torch.empty_like(o) for o in outs]
            call(new, eager)
            side.synchronize()
            for a, b in zip(got, eager):
                assert torch.equal(a, b), name


def test_two_streams_match_sequential(cuda):
    import torch

    rng = np.random.default_rng(7)
    a_cases = _cases(torch, cuda, rng)
    b_cases = _cases(torch, cuda, rng)
    s1, s2 = torch.cuda.Stream(cuda), torch.cuda.Stream(cuda)
    main = torch.cuda.current_stream(cuda)
    s1.wait_stream(main)
    s2.wait_stream(main)
    for (_, ia, oa, ca), (_, ib, ob, cb) in zip(a_cases, b_cases):
        with torch.cuda.stream(s1):
            ca(ia, oa)
        with torch.cuda.stream(s2):
            cb(ib, ob)
    s1.synchronize()
    s2.synchronize()
    concurrent = [[o.clone() for o in c[2]] for c in a_cases + b_cases]
    for name, ins, outs, call in a_cases + b_cases:
        call(ins, outs)
    main.synchronize()
    for (name, _, outs, _), want in zip(a_cases + b_cases, concurrent):
        for a, b in zip(outs, want):
            assert torch.equal(a, b), name
