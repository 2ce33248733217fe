"""Generate the golden fixtures for the GDN parity tests from the REFERENCE'S OWN CODE.

Run in a container where the reference tree is mounted (its path is given by
``--ref`` or the ``KAIROS_REF`` environment variable); the GPU box never runs
this script, it only reads the committed ``*.pt`` files.

Two reference implementations are executed on CPU in fp32:

1. ``naive_recurrent_gated_delta_product`` from
   ``kairos/third_party/fla/ops/gated_delta_product/naive.py:4-36``, imported
   by file path (it ignores ``scale``, so q is passed pre-scaled by K^-1/2,
   and q/k are passed L2-normalised, as the reference's own benchmark
   ``kairos_ext/bench_gdn_recurrent.py:62-74`` does).
2. The reference's Triton ``chunk_gated_delta_rule``
   (``kairos/third_party/fla/ops/gated_delta_rule/chunk.py:216-323``) under
   ``TRITON_INTERPRET=1`` with ``use_qk_l2norm_in_kernel=True``.  Four
   harness shims make the vendored package import and run on a CPU:
   a stub ``kairos.modules.utils`` (the real one imports video libraries),
   a no-op ``torch.cpu.device`` context (``fla/utils.py:158-160``), an
   autotuner whose benchmark returns constants (no GPU to time on), and
   re-bound ``exp/exp2/log/log2`` aliases in every loaded FLA module (the
   interpreter does not patch aliases captured at import, ``fla/ops/utils/op.py:16-20``).
   Nothing under the reference tree is modified.

Each fixture holds the inputs (bf16-representable fp32 values so that the GPU
path sees exactly the same numbers), both reference outputs and final states.
"""
from __future__ import annotations

import argparse
import contextlib
import importlib.util
import os
import sys
import types
from pathlib import Path

os.environ['TRITON_INTERPRET'] = '1'   # must precede the first triton import

import torch  # noqa: E402
import torch.nn.functional as F  # noqa: E402
import triton  # noqa: E402
import triton.language as tl  # noqa: E402


@triton.jit
def _exp(x):
    return tl.exp(x)


@triton.jit
def _exp2(x):
    return tl.math.exp2(x)


@triton.jit
def _log(x):
    return tl.log(x)


@triton.jit
def _log2(x):
    return tl.log2(x)


HERE = Path(__file__).resolve().parent


def gen_inputs(B, T, H, K, V, seed, g_scale=1.0, h0=False):
    """Seeded inputs with the distributions BASELINE config 0 specifies:
    q,k,v ~ N(0,1) drawn in that order; beta = sigmoid(N(0,1));
    g = -softplus(N(0,1)); q,k, v, beta rounded to bf16 values."""
    gen = torch.Generator().manual_seed(seed)
    q = torch.randn(B, T, H, K, generator=gen)
    k = torch.randn(B, T, H, K, generator=gen)
    v = torch.randn(B, T, H, V, generator=gen)
    beta = torch.randn(B, T, H, generator=gen).sigmoid()
    g = -F.softplus(torch.randn(B, T, H, generator=gen)) * g_scale
    q, k, v, beta = (x.bfloat16().float() for x in (q, k, v, beta))
    init = torch.randn(B, H, K, V, generator=gen) * 0.1 if h0 else None
    return q, k, v, g, beta, init


def load_naive(ref: Path):
    p = ref / 'kairos/third_party/fla/ops/gated_delta_product/naive.py'
    spec = importlib.util.spec_from_file_location('ref_naive_gdp', p)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.naive_recurrent_gated_delta_product


def load_triton_chunk(ref: Path):
    sys.path.insert(0, str(ref))
    stub = types.ModuleType('kairos.modules.utils')
    stub.FLAGS_KAIROS_CUDA_SM = 90
    stub.FLAGS_KAIROS_IS_METAX = False
    stub.FLAGS_KAIROS_PLAT_DEVICE = 'cuda'
    sys.modules['kairos.modules.utils'] = stub
    torch.cpu.device = lambda i: contextlib.nullcontext()
    triton.runtime.autotuner.Autotuner._bench = lambda self, *a, config=None, **k: [1.0, 1.0, 1.0]
    from kairos.third_party.fla.ops.gated_delta_rule.chunk import chunk_gated_delta_rule
    for name, m in list(sys.modules.items()):
        if name.startswith('kairos.third_party.fla') and m is not None:
            for a, f in (('exp', _exp), ('exp2', _exp2), ('log', _log), ('log2', _log2)):
                if hasattr(m, a):
                    setattr(m, a, f)
    return chunk_gated_delta_rule


CASES = [
    # name, B, T, H, K, V, seed, g_scale, h0
    ('cfg0', 1, 1024, 4, 128, 128, 0, 1.0, False),
    ('t1', 1, 1, 2, 128, 128, 11, 1.0, False),
    ('t63', 1, 63, 2, 128, 128, 12, 1.0, False),
    ('t64', 1, 64, 2, 128, 128, 13, 1.0, False),
    ('t65', 1, 65, 2, 128, 128, 14, 1.0, True),
    ('t1000', 1, 1000, 2, 128, 128, 15, 1.0, True),
    ('slowdecay', 1, 512, 2, 128, 128, 16, 0.01, False),
    ('b2', 2, 130, 2, 128, 128, 17, 1.0, True),
    ('k128v256', 1, 200, 2, 128, 256, 18, 1.0, True),
    ('k256v512', 1, 130, 1, 256, 512, 19, 1.0, True),
]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--ref', default=os.environ.get('KAIROS_REF', ''))
    ap.add_argument('--only', default='')
    args = ap.parse_args()
    ref = Path(args.ref)
    assert (ref / 'kairos').is_dir(), 'pass --ref <reference tree>'
    torch.set_num_threads(os.cpu_count())
    naive = load_naive(ref)
    chunk = load_triton_chunk(ref)
    for name, B, T, H, K, V, seed, gs, h0 in CASES:
        if args.only and name not in args.only.split(','):
            continue
        q, k, v, g, beta, init = gen_inputs(B, T, H, K, V, seed, gs, h0)
        qn = F.normalize(q, dim=-1, eps=0) * K ** -0.5
        kn = F.normalize(k, dim=-1, eps=0)
        with torch.no_grad():
            o_naive, s_naive = naive(qn, kn, v, g, beta, None, None,
                                     initial_state=None if init is None else init.clone(),
                                     output_final_state=True)
            o_tri, s_tri = chunk(q, k, v, g, beta, initial_state=init, output_final_state=True,
                                 use_qk_l2norm_in_kernel=True)
        d_o = ((o_naive - o_tri).abs().max() / o_naive.abs().max()).item()
        d_s = ((s_naive - s_tri).abs().max() / s_naive.abs().max()).item()
        print(f'{name}: naive vs triton-interpreter  o max-rel {d_o:.2e}  state max-rel {d_s:.2e}')
        assert d_o < 1e-4 and d_s < 1e-4, name
        # inputs are bf16-exact, so they are stored as bf16; the naive output of
        # the large cases is stored in bf16 to keep fixtures small (the Triton
        # output and both states stay fp32).
        o_n = o_naive.float()
        if o_n.numel() > 200000:
            o_n = o_n.bfloat16()
        torch.save(dict(q=q.bfloat16(), k=k.bfloat16(), v=v.bfloat16(), g=g, beta=beta.bfloat16(),
                        h0=init, o_naive=o_n, s_naive=s_naive.float(),
                        o_triton=o_tri.float(), s_triton=s_tri.float(),
                        meta=dict(B=B, T=T, H=H, K=K, V=V, seed=seed, g_scale=gs,
                                  agree_o=d_o, agree_s=d_s, agree=True)),
                   HERE / f'gdn_{name}.pt')


if __name__ == '__main__':
    main()
