"""The allocation-free SmoothQuant linear, svla_sq_linear_w8a8_static_scratch.

It is for callers that cannot allocate device memory -- a fixed-rate control loop that must not allocate
after start-up, or a binding that only holds the pointers it was given.  Its scratch is a fixed 4 MiB
array inside the library instead of a caller workspace.  The file name sorts last so that a run stopping at
the first failure (pytest -x) has already run every other test when this one runs.

Checked through the C ABI: two calls in a row, each on a different input, give exactly the output of
svla_sq_linear_w8a8 (the workspace entry point) -- the same kernels run, so the tolerance is zero -- and
leave the device's free memory unchanged (nothing is allocated per call); a call whose int8 activations would
not fit is refused with status 1 before any GPU work.
"""

import pytest
import torch

from smolvla_mujoco_libero_b200 import _lib, ops, synthetic

CAPACITY = 4 << 20


def _call(lib, x, smooth, a, qw, ws, bias, y):
    m, k = x.shape
    return lib.svla_sq_linear_w8a8_static_scratch(
        x.data_ptr(), smooth.data_ptr(), float(a), qw.data_ptr(), ws.data_ptr(),
        None if bias is None else bias.data_ptr(), m, qw.shape[0], k, y.data_ptr(),
        torch.cuda.current_stream().cuda_stream)


@pytest.mark.gpu
def test_static_scratch_entry_matches_workspace_entry_on_two_calls():
    lib = _lib.lib()
    dev = "cuda"
    case = synthetic.smoothquant_linear_case(seed=4321, with_bias=True)      # M 177, K 960, N 2560
    other = synthetic.smoothquant_linear_case(seed=8765, m=300, with_bias=True)
    smooth = (torch.rand(960, generator=synthetic.generator(9)) * 2 + 0.25).to(dev)
    qw, ws = ops.pack_weight_i8(case.weight.to(dev), smooth)
    bias = case.bias.to(dev)
    inputs = [(case.x.to(dev), 0.011), (other.x.to(dev), 0.017)]
    refs = [ops.sq_linear_w8a8(x, smooth, a, qw, ws, bias) for x, a in inputs]
    outs = [torch.full_like(r, float("nan")) for r in refs]
    # a first call looks up the array's device address; after it, calls must not change the free memory
    assert _call(lib, inputs[0][0], smooth, inputs[0][1], qw, ws, bias, outs[0]) == 0, lib.svla_last_error()
    torch.cuda.synchronize()
    outs[0].fill_(float("nan"))
    torch.cuda.synchronize()
    free0, allocated0 = torch.cuda.mem_get_info()[0], torch.cuda.memory_allocated()
    for (x, a), y in zip(inputs, outs):
        rc = _call(lib, x, smooth, a, qw, ws, bias, y)
        assert rc == 0, lib.svla_last_error()
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0
    assert torch.cuda.memory_allocated() == allocated0
    for y, ref in zip(outs, refs):
        assert torch.equal(y, ref)
    assert _lib.device_error() == 0


@pytest.mark.gpu
def test_static_scratch_entry_rejects_activations_beyond_its_array():
    lib = _lib.lib()
    m, k, n = 4097, 1024, 64                       # 4097 * 1024 int8 bytes > 4 MiB
    assert m * k > CAPACITY
    x = torch.zeros(m, k, dtype=torch.bfloat16, device="cuda")
    smooth = torch.ones(k, device="cuda")
    qw = torch.zeros(n, k, dtype=torch.int8, device="cuda")
    ws = torch.ones(n, device="cuda")
    y = torch.zeros(m, n, dtype=torch.bfloat16, device="cuda")
    assert _call(lib, x, smooth, 0.1, qw, ws, None, y) == 1
    assert b"exceeds the fixed scratch" in lib.svla_last_error()
