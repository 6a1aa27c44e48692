"""vc4_matvec_s_noalloc: GPU::matvec_s for callers that cannot allocate.

A caller whose device memory belongs to its own pool, or whose thread must not
risk the synchronisation an allocation can cause, passes its own device input
and output buffers; the library keeps its scratch in a static device array.
Checked here through the C ABI against vc4_matvec_s (the allocating entry
point) on two calls in a row per matrix, with the same exact-equality
tolerance the other matvec parity tests use, plus the size limit.

This file sorts last so that a `-x` run has executed every other test before
it; it also passes on its own in a fresh process.
"""
import ctypes as C

import numpy as np
import pytest

import vc4b200


def _call(model, which, layer, expert, x, check_memory=False):
    """The no-alloc call through the C ABI on caller-owned device buffers.
    With check_memory the driver's free device memory is read right before
    and after the call (buffers already allocated) and must not change."""
    import torch
    L = vc4b200.lib()
    w = vc4b200.MATS[which]
    rows = model.matvec_s(which, x, layer=layer, expert=expert).shape[0]
    dx = torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
    dout = torch.full((rows,), float("nan"), dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    rc = L.vc4_matvec_s_noalloc(model._h, w, layer, expert, C.c_void_p(dx.data_ptr()),
                                C.c_void_p(dout.data_ptr()), C.c_void_p(stream))
    assert rc == 0, L.vc4_last_error().decode()
    torch.cuda.synchronize()
    if check_memory:
        assert torch.cuda.mem_get_info()[0] == free0, "%s: device memory changed across the call" % which
    return dout.cpu().numpy()


@pytest.mark.gpu
@pytest.mark.parametrize("key", ["tiny_q8", "tiny_q4", "tiny_t3", "tiny_moe_q4", "tiny_flat_q8"])
def test_noalloc_matvec_matches_allocating_entry_point(tiny_paths, key):
    gpu = vc4b200.GPU(0)
    model = vc4b200.Model(gpu, tiny_paths[key])
    rng = np.random.default_rng(11)
    info = model.info
    # each matrix's own input width: wo reads the heads' outputs, w2 the FFN
    # hidden vector (the widest input), the rest the model width
    cols_of = {"wo": info.heads * info.head_dim, "w2": info.ffn_width}
    cases = [("qkv", 0, 0), ("wo", 1, 0), ("w1", 1, 0), ("logits", 0, 0)]
    if info.experts:
        cases += [("router", 0, 0), ("w3", 0, 3)]
    if not info.ffn_chunked:
        # a chunked FFN's w2 is two column halves, which matvec_s never draws whole
        cases += [("w2", 1, 2 if info.experts else 0)]
    for which, layer, expert in cases:
        cols = cols_of.get(which, info.dim)
        for call in range(2):                       # two calls in a row share the scratch
            x = (rng.integers(-3000, 3000, size=cols) / 256.0 * (0.01 if call else 1.0)).astype(np.float32)
            want = model.matvec_s(which, x, layer=layer, expert=expert)
            # from the second call on a device nothing may be allocated
            got = _call(model, which, layer, expert, x, check_memory=call == 1)
            assert np.array_equal(got, want), "%s layer %d call %d" % (which, layer, call)


@pytest.mark.gpu
def test_noalloc_rejects_matrices_beyond_the_scratch(tiny_paths, tmp_path):
    """A matrix wider or taller than the static array is refused up front."""
    import torch
    from vc4b200 import mmcf_writer, synth
    shape = synth.Shape("tall-vocab", 64, 2112, 1, 4, 2, 90000, 1e6, True)
    path = str(tmp_path / "tall.mmcf")
    with open(path, "wb") as f:
        f.write(mmcf_writer.pack(shape, synth.hf_tensors(shape, 3), "q8", 64))
    gpu = vc4b200.GPU(0)
    model = vc4b200.Model(gpu, path)
    dx = torch.zeros(64, dtype=torch.float32, device="cuda")
    dout = torch.zeros(90000, dtype=torch.float32, device="cuda")
    L = vc4b200.lib()
    rc = L.vc4_matvec_s_noalloc(model._h, 6, 0, 0, C.c_void_p(dx.data_ptr()), C.c_void_p(dout.data_ptr()), None)
    assert rc == 1 and b"scratch limit" in L.vc4_last_error()
