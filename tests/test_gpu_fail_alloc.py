"""Failure detection on the host side of b2_load: an injected device
allocation failure (b2_debug_fail_alloc; nothing faults the GPU) must surface
as B2_ERR_OOM and leave no device memory behind."""
import pytest

import b2decode

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("nth", [1, 2])
def test_load_allocation_failure_leaks_nothing(built_lib, tiny_gguf, nth):
    import torch
    torch.cuda.init()
    m0 = b2decode.Model(tiny_gguf)  # warm the context and the library's statics
    m0.close()
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    b2decode.debug_fail_alloc(nth)  # 1: the arena, 2: the upload buffer
    try:
        with pytest.raises(b2decode.B2Error) as ei:
            b2decode.Model(tiny_gguf)
    finally:
        b2decode.debug_fail_alloc(0)
    assert b2decode.ERRORS[ei.value.code] == "OOM"
    assert "allocation" in str(ei.value)
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0
    m = b2decode.Model(tiny_gguf)  # the next load is unaffected
    assert m.forward_argmax([1, 2, 3]) >= 0
    m.close()
