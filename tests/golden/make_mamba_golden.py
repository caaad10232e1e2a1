"""Golden vectors for the Mamba-2 oracle, made with transformers' NemotronHMamba2Mixer
(an independent implementation of the same layer; the reference's own mlx-lm path cannot run
here). Run from the repo root: python tests/golden/make_mamba_golden.py

A tiny fp32 mixer (hidden 32, 4 heads x 8, 2 groups, state 16, conv 4, no dt clamp) with
seeded weights runs its SSD path over 12 tokens from a zero state in ONE chunk (chunk_size 16):
inside a chunk that path is the exact quadratic form of the recurrence. (Across chunk
boundaries this transformers version's inter-chunk term disagrees with the recurrence and
with its own single-chunk result, so the fixture stays inside one chunk.) The file stores the
weights, the inputs and the outputs. tests/test_oracle.py checks oracle/mamba.py's
row-by-row recurrence against it.
"""
import os

import numpy as np
import torch
from transformers.models.nemotron_h.configuration_nemotron_h import NemotronHConfig
from transformers.models.nemotron_h.modeling_nemotron_h import NemotronHMamba2Mixer

HERE = os.path.dirname(os.path.abspath(__file__))


def main():
    torch.manual_seed(1234)
    cfg = NemotronHConfig(hidden_size=32, mamba_num_heads=4, mamba_head_dim=8, n_groups=2, ssm_state_size=16,
                          conv_kernel=4, chunk_size=16, time_step_min=0.0, time_step_limit=(0.0, float("inf")),
                          layer_norm_epsilon=1e-5, use_conv_bias=True, use_bias=False)
    m = NemotronHMamba2Mixer(cfg, layer_idx=0).float().eval()
    with torch.no_grad():
        for prm in m.parameters():
            prm.copy_(torch.randn_like(prm) * 0.3)
        m.A_log.copy_(torch.log(torch.linspace(0.5, 2.0, 4)))
        m.dt_bias.copy_(torch.linspace(-1.0, 0.5, 4))
        m.norm.weight.copy_(1.0 + 0.1 * torch.randn(32))
        x = torch.randn(1, 12, 32)
        out = m.torch_forward(x, cache_params=None)
    np.savez_compressed(os.path.join(HERE, "mamba_mixer.npz"), x=x[0].numpy(), out=out[0].numpy(),
                        in_proj=m.in_proj.weight.detach().numpy(), conv_w=m.conv1d.weight.detach()[:, 0].numpy(),
                        conv_b=m.conv1d.bias.detach().numpy(), A_log=m.A_log.detach().numpy(),
                        D=m.D.detach().numpy(), dt_bias=m.dt_bias.detach().numpy(),
                        norm_w=m.norm.weight.detach().numpy(), out_proj=m.out_proj.weight.detach().numpy(),
                        dims=np.array([4, 8, 2, 16]), eps=np.array([1e-5]))
    print("wrote mamba_mixer.npz")


if __name__ == "__main__":
    main()
