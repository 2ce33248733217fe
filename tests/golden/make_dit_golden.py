"""Golden fixture for the DiT block structure, produced by the REFERENCE'S OWN
``DiTBlock`` (``kairos/modules/dits/kairos_dit.py:727-972``) on CPU in fp32.

Run in a container where the reference tree is mounted (``--ref`` or the
``KAIROS_REF`` environment variable); the GPU box never runs this script.

The block is built with softmax attention (``use_linear_attn=False``,
``dilated_length=1``): on a machine without flash-attn kernels for the inputs'
device, ``flash_attention`` takes its own SDPA branch (``kairos_dit.py:266-276``),
which ignores the window, i.e. full attention -- the attention of the
benchmark.  Harness shims only (nothing under the reference tree changes):

* stub modules for the package-level imports the block does not use on this
  path: ``kairos.apis.builder`` (registry decorator), ``kairos.modules.utils``
  (flags, ``parallel_state``), ``kairos.modules.utils.tp_utils``, the
  tensor-parallel GDN layer, the FLA cache and ``fla`` itself;
* ``apex.normalization.fused_layer_norm.FusedRMSNorm`` as its published math
  (y = x * rsqrt(mean(x^2) + eps) * weight over the last dimension, fp32);
* the module's flash-attn availability flags set to False after import, so
  the CPU tensors take the SDPA branch (flash-attn 2.8 is installed here but
  runs on CUDA tensors only).

The fixture holds the block's state dict, its inputs (x, context, t_mod, the
3-D RoPE factors and the grid) and its output.
"""
from __future__ import annotations

import argparse
import importlib.util
import os
import sys
import types
from pathlib import Path

import torch
import torch.nn as nn

OUT = Path(__file__).resolve().parent / 'dit_block_attn.pt'


class _FusedRMSNorm(nn.Module):
    def __init__(self, normalized_shape, eps=1e-5, elementwise_affine=True):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(normalized_shape))

    def forward(self, x):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps) * self.weight).to(x.dtype)


def _stub(name, **attrs):
    m = types.ModuleType(name)
    m.__dict__.update(attrs)
    sys.modules[name] = m
    return m


def load_reference_dit(ref: Path):
    dits = ref / 'kairos' / 'modules' / 'dits'
    _stub('apex')
    _stub('apex.normalization')
    _stub('apex.normalization.fused_layer_norm', FusedRMSNorm=_FusedRMSNorm)
    _stub('kairos').__path__ = []
    _stub('kairos.modules').__path__ = []
    _stub('kairos.modules.dits').__path__ = [str(dits)]
    ps = types.SimpleNamespace(get_context_parallel_rank=lambda: 0, get_context_parallel_world_size=lambda: 1,
                               get_context_parallel_group=lambda: None)
    _stub('kairos.modules.utils', FLAGS_KAIROS_CUDA_SM=0, FLAGS_KAIROS_IS_METAX=False, parallel_state=ps).__path__ = []
    _stub('kairos.modules.utils.tp_utils', build_tp_chunk_list=None, all2all_seq_to_head=None,
          all2all_head_to_seq=None, _gather_input_sp=None, _distribute_input_sp=None)

    class _Registry:
        def register_module(self, *a, **k):
            return lambda cls: cls
    _stub('kairos.apis').__path__ = []
    _stub('kairos.apis.builder', DITS=_Registry())
    for n in ('kairos.third_party', 'kairos.third_party.fla', 'kairos.third_party.fla.layers',
              'kairos.third_party.fla.models'):
        _stub(n).__path__ = []
    _stub('kairos.third_party.fla.layers.gated_deltanet_with_tp', GatedDeltaNet=None)
    _stub('kairos.third_party.fla.models.utils', Cache=None)
    _stub('fla').__path__ = []
    _stub('fla.layers', GatedDeltaNet=None)
    _stub('fla.utils', autotune_cache_kwargs={})
    spec = importlib.util.spec_from_file_location('kairos.modules.dits.kairos_dit', dits / 'kairos_dit.py')
    mod = importlib.util.module_from_spec(spec)
    mod.__package__ = 'kairos.modules.dits'
    sys.modules[spec.name] = mod
    spec.loader.exec_module(mod)
    mod.FLASH_ATTN_2_AVAILABLE = False
    mod.FLASH_ATTN_3_AVAILABLE = False
    mod.SAGE_ATTN_AVAILABLE = False
    return mod


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--ref', default=os.environ.get('KAIROS_REF', ''))
    args = ap.parse_args()
    if not args.ref:
        raise SystemExit('pass --ref <reference checkout> or set KAIROS_REF')
    kd = load_reference_dit(Path(args.ref))
    torch.manual_seed(11)
    dim, heads, ffn, eps = 256, 2, 512, 1e-6
    blk = kd.DiTBlock(False, dim, heads, ffn, eps, use_linear_attn=False, dilated_length=1, window_size=3,
                      block_idx=0).float().eval()
    with torch.no_grad():
        for name, p in blk.named_parameters():
            if name == 'modulation':
                continue                               # keeps its randn / sqrt(dim) init
            if name.endswith('norm_q.weight') or name.endswith('norm_k.weight') or name == 'cross_attn_norm.weight':
                p.uniform_(0.5, 1.5)
            else:
                p.normal_(0.0, 0.02 if p.dim() > 1 else 0.05)
    f, h, w = 4, 4, 4
    T = f * h * w
    hd = dim // heads
    fr = kd.precompute_freqs_cis_3d(hd)
    freqs = torch.cat([fr[0][:f].view(f, 1, 1, -1).expand(f, h, w, -1),
                       fr[1][:h].view(1, h, 1, -1).expand(f, h, w, -1),
                       fr[2][:w].view(1, 1, w, -1).expand(f, h, w, -1)], dim=-1).reshape(T, 1, -1)
    x = torch.randn(1, T, dim)
    context = torch.randn(1, 16, dim)
    t_mod = torch.randn(1, 6, dim) * 0.1
    with torch.no_grad():
        y = blk(x.clone(), context, t_mod, freqs, (f, h, w))
    torch.save(dict(state_dict={k: v.clone() for k, v in blk.state_dict().items()}, x=x, context=context,
                    t_mod=t_mod, grid=(f, h, w), dim=dim, heads=heads, ffn_dim=ffn, eps=eps, out=y), OUT)
    print(f'wrote {OUT} (out std {float(y.std()):.4f})')


if __name__ == '__main__':
    main()
