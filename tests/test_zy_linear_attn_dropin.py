"""turbomoe.linear_attn.install on Hugging Face's Qwen3_5MoeGatedDeltaNet,
against the unmodified module, both on the GPU.

The prompt runs the module's own chunked forward on both sides; the decode
steps run tm_gdn_decode on one side and the module's torch path on the
other, with the same projection GEMMs around them.  Bars: the layer-output
tolerance on every step's output (max-abs 2e-2, cosine 0.9995), the conv
state bit-exact, and the fp32 recurrent state after the last step within
max-abs 5e-3 and ||dS|| / ||S|| <= 2e-2.  The state bar allows one bf16 ulp
of a head's gate scalars between the two paths (a one-ulp difference of beta
scales that head's update by 2^-8): measured on B200 after a decode
step with the projections on [B, H] views, one value head of four moved by a
uniform factor of 1.004 (max-abs 5.7e-4, relative 3.3e-3) while the others
agreed to 2e-5.  The kernel's own precision is covered against the oracle in
tests/test_gpu_gdn.py.
"""
import copy

import pytest
import torch

pytestmark = pytest.mark.gpu


class _StateCache:
    """The conv/recurrent state interface of the reference's Qwen35Cache
    (cache/qwen35_cache.py:7-40), enough for the module's forward."""

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


def test_gdn_dropin_vs_hf_module_on_gpu():
    from transformers import Qwen3_5MoeTextConfig
    from transformers.models.qwen3_5_moe import modeling_qwen3_5_moe as M
    from turbomoe import linear_attn
    cfg = Qwen3_5MoeTextConfig(hidden_size=256, linear_num_key_heads=2, linear_num_value_heads=4,
                               linear_key_head_dim=128, linear_value_head_dim=128, linear_conv_kernel_dim=4)
    torch.manual_seed(5)
    ref = M.Qwen3_5MoeGatedDeltaNet(cfg, layer_idx=0)
    with torch.no_grad():
        ref.norm.weight.copy_(1.0 + 0.1 * torch.randn(128))
    ref = ref.to("cuda", torch.bfloat16).eval()
    ours = copy.deepcopy(ref)
    linear_attn.install(ours)
    ca, cb = _StateCache(), _StateCache()
    g = torch.Generator().manual_seed(6)
    with torch.no_grad():
        x = torch.randn(2, 5, 256, generator=g).to("cuda", torch.bfloat16)
        ya, yb = ref(x, cache_params=ca), ours(x, cache_params=cb)
        assert float((ya.float() - yb.float()).abs().max()) <= 1e-2    # the module's own prompt path
        for _ in range(3):
            x = torch.randn(2, 1, 256, generator=g).to("cuda", torch.bfloat16)
            ya, yb = ref(x, cache_params=ca), ours(x, cache_params=cb)
            assert yb.shape == ya.shape and yb.dtype == ya.dtype
            a, b = ya.float().flatten(), yb.float().flatten()
            cos = float(torch.nn.functional.cosine_similarity(a, b, dim=0))
            assert float((a - b).abs().max()) <= 2e-2 and cos >= 0.9995, cos
            assert torch.equal(ca.layers[0].conv_states, cb.layers[0].conv_states)
    want = ca.layers[0].recurrent_states.float()
    diff = cb.layers[0].recurrent_states - want
    d, rel = float(diff.abs().max()), float(diff.norm() / want.norm())
    assert d <= 5e-3 and rel <= 2e-2, (d, rel)
