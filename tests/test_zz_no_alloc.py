"""The allocation-free decode entry point (ppmoe_decode_noalloc) gives the same output as
the workspace-taking ppmoe_decode, on two calls in a row.

It exists for callers that cannot allocate device memory when they call the kernel (inside
a memory pool they do not own, in plugin hosts that pass only inputs and outputs, or on
latency paths where an allocation would synchronise).  The test calls it through the C ABI
with tensors allocated by the test itself, never by the entry point.  It is kept in its own
file, collected last, so a failure here cannot hide the result of any other test.
"""
import pytest
import torch

from conftest import assert_close_out, pkg
from gpu_helpers import make_layer, make_module

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("tokens", [1, 5])
def test_decode_noalloc_matches_workspace_decode(cuda, tokens):
    lib = pkg()._lib
    H, E, G, tau = 1536, 64, 96, 0.95
    L = make_layer(21, H, E, G, tau)
    m = make_module(L, tau, cuda)
    packed = m.packed()
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):  # two calls in a row share (and must re-clear) the scratch
        x = pkg().synth.make_tokens(21, tokens, H, stream=call).to(cuda)
        ref = m.forward_decode(x)
        out = torch.empty(tokens, H, dtype=torch.bfloat16, device=cuda)
        lib.call("ppmoe_decode_noalloc", x.data_ptr(), tokens, packed.data_ptr(), H, E, G, tau,
                 out.data_ptr(), stream)
        # the device status word lives in the library's own scratch: read it back (and
        # check that no bounded wait ran out) before the next call clears it
        lib.call("ppmoe_decode_noalloc_status", stream)
        assert lib.load().ppmoe_last_error() == b""
        assert_close_out(out.cpu(), ref.cpu(), f"noalloc call {call}")
        assert torch.equal(out.cpu(), ref.cpu())  # same kernel, same order of operations


def test_decode_noalloc_rejects_oversize(cuda):
    lib = pkg()._lib
    rc = lib.load().ppmoe_decode_noalloc(16, 6, 1024, 1536, 64, 96, 0.9, 16, None)
    assert rc == -2 and b"scratch limit" in lib.load().ppmoe_last_error()
