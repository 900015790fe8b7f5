"""The product path has no CPU fallback: on a machine without a GPU, creating a handle (here
through __graft_entry__.smoke, which builds a tiny model and runs it on device 0) fails in the
library with ECUDA instead of computing anything on the host."""
import pytest
import torch

from smelt_b200._ffi import Gpt2qError


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the behaviour without a GPU")
def test_smoke_fails_loudly_without_a_gpu():
    import __graft_entry__ as entry

    with pytest.raises(Gpt2qError) as e:
        entry.smoke()
    assert e.value.code == -3
