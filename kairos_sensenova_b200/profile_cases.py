"""Small, self-contained cases of the hot-path operators for profilers.

    python -m kairos_sensenova_b200.profile_cases attn S H   # attention_fp8 on attn_inputs(1, S, H, 128, seed=1)
    python -m kairos_sensenova_b200.profile_cases gdn  T H   # chunk_gated_delta_rule on gdn_inputs(1, T, H, 128, 128, seed=0)
    python -m kairos_sensenova_b200.profile_cases prologue T H  # gdn_prologue on a fused [T, 3*H*128 + 2H (+pad)] projection
    python -m kairos_sensenova_b200.profile_cases resln T C     # residual_ln_mod on [T, C] bf16 rows
    python -m kairos_sensenova_b200.profile_cases dit L         # one eager DiT step (config 4 shapes, L blocks)

Each runs the operator twice (warm) on synthetic seeded inputs and exits, so an
``ncu -k <kernel> -s <n> -c 1`` capture sees a handful of launches of a
bounded size.
"""
from __future__ import annotations

import sys

import torch


def main(argv):
    what = argv[1] if len(argv) > 1 else 'attn'
    n = int(argv[2]) if len(argv) > 2 else 8192
    h = int(argv[3]) if len(argv) > 3 else 8
    if what == 'attn':
        from .attention import attention_fp8
        from .inputs import attn_inputs
        q, k, v = attn_inputs(1, n, h, 128, seed=1)
        for _ in range(2):
            attention_fp8(q, k, v, h)
    elif what == 'gdn':
        from .gated_delta_rule import chunk_gated_delta_rule
        from .inputs import gdn_inputs
        q, k, v, g, beta = gdn_inputs(1, n, h, 128, 128, seed=0)
        for _ in range(2):
            chunk_gated_delta_rule(q, k, v, g, beta, output_final_state=True, use_qk_l2norm_in_kernel=True)
    elif what == 'prologue':
        from .fused_ops import gdn_prologue
        gen = torch.Generator(device='cuda')
        gen.manual_seed(0)
        C = (3 * h * 128 + 2 * h + 7) // 8 * 8
        proj = torch.randn(n, C, generator=gen, device='cuda').to(torch.bfloat16)
        w = torch.rand(h * 128, 4, generator=gen, device='cuda') - 0.5
        A_log, dtb = torch.zeros(h, device='cuda'), torch.zeros(h, device='cuda')
        s = lambda i: proj[:, i * h * 128:(i + 1) * h * 128]  # noqa: E731
        ab = 3 * h * 128
        for _ in range(2):
            gdn_prologue(s(0), s(1), s(2), proj[:, ab:ab + h], proj[:, ab + h:ab + 2 * h], w, w, w, A_log, dtb,
                         h, 1, n)
    elif what == 'resln':
        from .fused_ops import residual_ln_mod
        gen = torch.Generator(device='cuda')
        gen.manual_seed(0)
        x = torch.randn(n, h, generator=gen, device='cuda').to(torch.bfloat16)
        r = torch.randn(n, h, generator=gen, device='cuda').to(torch.bfloat16)
        vec = [torch.randn(h, generator=gen, device='cuda') for _ in range(3)]
        y = torch.empty_like(x)
        for _ in range(2):
            residual_ln_mod(x, r, vec[0], vec[1], vec[2], True, 1e-6, out=y)
    elif what == 'dit':
        from .dit import DiTConfig, KairosDiT
        cfg = DiTConfig(layers=int(argv[2]) if len(argv) > 2 else 30)
        model = KairosDiT(cfg)
        gen = torch.Generator(device='cuda')
        gen.manual_seed(2)
        lat = torch.randn(cfg.in_dim, *cfg.latent, generator=gen, device='cuda')
        ctx = torch.randn(cfg.text_len, cfg.text_dim, generator=gen, device='cuda')
        with torch.no_grad():
            model(lat, torch.tensor([500.0], device='cuda'), ctx)
    else:
        raise SystemExit(f'unknown case {what!r} (attn | gdn | prologue | resln | dit)')
    torch.cuda.synchronize()
    print('ok')


if __name__ == '__main__':
    main(sys.argv)
