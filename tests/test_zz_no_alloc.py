"""ceb_moe_ffn_static: the MoE block for callers that may not allocate device memory.

Such callers (a host whose GPU memory is owned by another allocator, a plugin that
only gets a stream, a path that cannot take cudaMalloc's synchronisation) call an
entry point whose scratch is a fixed array inside the library.  These tests call
it through the C ABI and check it against ceb_moe_ffn (caller-provided workspace)
on two calls in a row -- the second call finds the first call's leftovers in the
shared scratch -- and that oversized batches are refused.  Both entry points run
the same kernels on the same routing, so the outputs must be bit-identical.  The
second batch (666 expert rows after 1,400) ends inside a GEMM tile whose tail rows
still hold the first call's data, which must not reach the output.  After a
warm-up call, a further call must leave the device's free memory and torch's
allocator untouched: the entry point allocates nothing.  This file is collected
last on purpose; it also passes on its own in a fresh process.
"""
import numpy as np
import pytest

from crispembed_b200 import synth
from crispembed_b200.gguf_io import GGML_F32, GGML_Q8_0

pytestmark = pytest.mark.gpu


def _layer(binding, inp):
    return binding.MoELayer(inp.d, inp.n_experts, inp.top_k, inp.ffn, inp.router_wtype, inp.router_raw, inp.wtype,
                            inp.fc1_raw, inp.fc2_raw, inp.bias)


def test_static_matches_workspace_entry_twice(cuda):
    import torch
    from crispembed_b200 import binding
    # two different batches so the second call runs over the first call's scratch contents
    a = synth.make_moe_op_inputs(700, d=768, n_experts=8, top_k=2, ffn=3072, wtype=GGML_Q8_0,
                                 router_wtype=GGML_Q8_0, zipf_s=1.2, seed=21, with_bias=True)
    b = synth.make_moe_op_inputs(333, d=768, n_experts=8, top_k=2, ffn=3072, wtype=GGML_Q8_0,
                                 router_wtype=GGML_Q8_0, zipf_s=None, seed=21, with_bias=True)
    layer = _layer(binding, a)  # same weights (same seed) for both batches
    for inp in (a, b):
        T = inp.x.shape[0]
        x = torch.from_numpy(inp.x).to(cuda).to(torch.bfloat16)
        ws = torch.empty(layer.workspace_size(T), dtype=torch.uint8, device=cuda)
        y_ref = torch.empty((T, inp.d), dtype=torch.float32, device=cuda)
        layer.forward(x, y_ref, ws)
        y = torch.full((T, inp.d), float("nan"), dtype=torch.float32, device=cuda)
        layer.forward_static(x, y)
        binding.sync_check()
        r, g = y_ref.cpu().numpy(), y.cpu().numpy()
        assert np.isfinite(g).all()
        assert np.array_equal(g, r), np.abs(g - r).max()
    layer.close()


def test_static_call_allocates_nothing(cuda):
    import torch
    from crispembed_b200 import binding
    inp = synth.make_moe_op_inputs(500, d=768, n_experts=8, top_k=2, ffn=3072, wtype=GGML_Q8_0,
                                   router_wtype=GGML_Q8_0, zipf_s=None, seed=22, with_bias=True)
    layer = _layer(binding, inp)
    x = torch.from_numpy(inp.x).to(cuda).to(torch.bfloat16)
    y = torch.empty((inp.x.shape[0], inp.d), dtype=torch.float32, device=cuda)
    y2 = torch.empty_like(y)
    layer.forward_static(x, y)  # warm-up: the first call on a device looks the scratch up
    binding.sync_check()
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    stats0 = torch.cuda.memory_stats()
    layer.forward_static(x, y2)
    binding.sync_check()
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    stats1 = torch.cuda.memory_stats()
    assert free1 == free0, (free0, free1)
    for key in ("num_alloc_retries", "num_device_alloc", "num_device_free"):
        assert stats1.get(key, 0) == stats0.get(key, 0), key
    assert torch.equal(y, y2)
    layer.close()


def test_static_rejects_oversized_batch(cuda):
    import torch
    from crispembed_b200 import binding
    inp = synth.make_moe_op_inputs(8, d=256, n_experts=4, top_k=2, ffn=512, wtype=GGML_Q8_0,
                                   router_wtype=GGML_F32, zipf_s=None, seed=1)
    layer = _layer(binding, inp)
    lib = binding.load_library()
    T = 1
    while layer.workspace_size(T) <= (64 << 20):
        T *= 2
    x = torch.zeros((T, inp.d), dtype=torch.float32, device=cuda)
    y = torch.zeros((T, inp.d), dtype=torch.float32, device=cuda)
    with pytest.raises(binding.CrispEmbedError, match="static"):
        layer.forward_static(x, y)
    assert "scratch" in binding.last_error()
    # the refusal left nothing behind: a valid call still works
    small = torch.from_numpy(inp.x).to(cuda)
    out = torch.empty((inp.x.shape[0], inp.d), dtype=torch.float32, device=cuda)
    layer.forward_static(small, out)
    binding.sync_check()
    assert np.isfinite(out.cpu().numpy()).all()
    del lib
    layer.close()
