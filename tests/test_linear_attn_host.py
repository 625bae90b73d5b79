"""Host logic of turbomoe.linear_attn on the CPU (no kernel launches).

``install`` must leave prompts (more than one token, or no cached state) to
the module's own forward, and a decode call must reach tm_gdn_decode, which
refuses CPU tensors: there is no CPU fallback.
"""
import pytest
import torch

from turbomoe import linear_attn
from turbomoe._lib import TurboMoEError


class _StateCache:
    class _L:
        conv_states = None
        recurrent_states = None

    def __init__(self):
        self.layers = {0: self._L()}

    def has_previous_state(self, i):
        return self.layers[i].conv_states is not None and self.layers[i].recurrent_states is not None

    def update_conv_state(self, s, i):
        self.layers[i].conv_states = s

    def update_recurrent_state(self, s, i):
        self.layers[i].recurrent_states = s


def _module():
    from transformers import Qwen3_5MoeTextConfig
    from transformers.models.qwen3_5_moe import modeling_qwen3_5_moe as M
    cfg = Qwen3_5MoeTextConfig(hidden_size=256, linear_num_key_heads=1, linear_num_value_heads=2,
                               linear_key_head_dim=128, linear_value_head_dim=128, linear_conv_kernel_dim=4)
    torch.manual_seed(3)
    return M.Qwen3_5MoeGatedDeltaNet(cfg, layer_idx=0).eval()


def test_install_keeps_prompts_on_the_module_and_refuses_cpu_decode():
    ref, mod = _module(), _module()
    linear_attn.install(mod)
    ca, cb = _StateCache(), _StateCache()
    x = torch.randn(2, 5, 256)
    with torch.no_grad():
        ya, yb = ref(x, cache_params=ca), mod(x, cache_params=cb)
        assert torch.equal(ya, yb)                                   # the module's own chunked forward
        assert torch.equal(ca.layers[0].recurrent_states, cb.layers[0].recurrent_states)
        assert torch.equal(mod(x[:, :1]), ref(x[:, :1]))             # no cache: the module's forward
        with pytest.raises(TurboMoEError, match="CUDA"):
            mod(x[:, :1], cache_params=cb)                           # decode step: kernel only


def test_decode_step_rejects_non_decode_calls():
    step = linear_attn.GatedDeltaNetDecode(_module())
    with pytest.raises(TurboMoEError, match="one token"):
        step(torch.randn(1, 3, 256), _StateCache())
    with pytest.raises(TurboMoEError, match="one token"):
        step(torch.randn(1, 1, 256), _StateCache())                 # no cached state yet
