"""Models whose execution template the device does not run yet (LFM2 short conv, MoE) are refused
at load with LLMDOT_E_UNSUPPORTED: no CPU fallback and no silent wrong answer.  The check runs on
the host before anything is allocated."""
import pytest

from dotllm_b200 import synth
from dotllm_b200.native import CudaBackendError

pytestmark = pytest.mark.gpu

LLMDOT_E_UNSUPPORTED = -2


@pytest.mark.parametrize("name", ["micro-lfm2", "micro-moe", "micro-lfm2moe"])
def test_templates_not_on_the_device_are_refused(gpu, name):
    from dotllm_b200.engine import CudaModel
    path = synth.build_model(synth.get(name))
    with pytest.raises(CudaBackendError) as e:
        CudaModel.load(path)
    assert e.value.status == LLMDOT_E_UNSUPPORTED, e.value.message
