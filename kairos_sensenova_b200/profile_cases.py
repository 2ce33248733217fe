"""Small, self-contained cases of the hot-path operators for profilers.

    python -m kairos_sensenova_b200.profile_cases attn S H   # attention_fp8 on attn_inputs(1, S, H, 128, seed=1)
    python -m kairos_sensenova_b200.profile_cases gdn  T H   # chunk_gated_delta_rule on gdn_inputs(1, T, H, 128, 128, seed=0)

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
    else:
        raise SystemExit(f'unknown case {what!r} (attn | gdn)')
    torch.cuda.synchronize()
    print('ok')


if __name__ == '__main__':
    main(sys.argv)
