"""Golden fixture for the GatedDeltaNet branch of the reference's ``DiTBlock``
(``kairos/modules/dits/kairos_dit.py:727-972``), run on CPU in fp32: the block's
own single-device path, which walks the sequence in T/8 pieces through one FLA
``Cache`` (``:857-922``), then the gated residual, cross-attention and FFN.

Run in a container where the reference tree is mounted (``--ref`` or
``KAIROS_REF``); the GPU box only reads the committed fixture.  Harness shims
(nothing under the reference tree changes):

* the Triton kernels of the vendored fla layer run under ``TRITON_INTERPRET=1``
  with the shims of ``make_golden.py`` / ``make_layer_golden.py`` (math-function
  stand-ins, SM count 148);
* ``DiTBlock`` imports ``GatedDeltaNet`` from the pip ``fla`` package, which is
  not installed here: the reference's vendored copy
  (``kairos/third_party/fla/layers/gated_deltanet.py``) stands in for it, and
  ``fla_Cahce`` is the vendored ``kairos/third_party/fla/models/utils.py`` Cache;
* ``torch.compile`` (the decorator on ``DiTBlock.forward``) is replaced by the
  identity, so the block runs eagerly;
* ``apex``'s FusedRMSNorm, the registry, the tensor-parallel utilities and
  ``parallel_state`` as in ``make_dit_golden.py``;
* after construction the block's ``gated_delta`` is rebuilt with head_dim 128 and
  expand_v 1 (the benchmark's 24 x 128 layout; ``DiTBlock`` passes fla's
  defaults, 256 / 2, which the kernels also support but the model does not use).

The fixture holds the block's state dict, its inputs, the GDN branch's input
and output (gathered over the T/8 pieces) and the block output.
"""
from __future__ import annotations

import argparse
import importlib.util
import os
import sys
import types
from pathlib import Path

os.environ['TRITON_INTERPRET'] = '1'   # must precede the first triton import

import torch  # noqa: E402

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import make_golden as mg  # noqa: E402
from make_dit_golden import _FusedRMSNorm, _stub  # noqa: E402

OUT = HERE / 'dit_block_gdn.pt'


def load(ref: Path):
    mg.load_triton_chunk(ref)                      # ref on sys.path, Triton interpreter shims
    utils = sys.modules['kairos.modules.utils']
    utils.__path__ = []
    utils.parallel_state = types.SimpleNamespace(get_context_parallel_rank=lambda: 0,
                                                 get_context_parallel_world_size=lambda: 1,
                                                 get_context_parallel_group=lambda: None)
    utils.FLAGS_KAIROS_IS_METAX = False
    _stub('kairos.modules.utils.tp_utils', build_tp_chunk_list=None, all2all_seq_to_head=None,
          all2all_head_to_seq=None, _gather_input_sp=None, _distribute_input_sp=None)
    from kairos.third_party.fla.layers.gated_deltanet import GatedDeltaNet
    from kairos.third_party.fla.models.utils import Cache
    for name, m in list(sys.modules.items()):
        if name.startswith('kairos.third_party.fla') and m is not None:
            for a, f in (('exp', mg._exp), ('exp2', mg._exp2), ('log', mg._log), ('log2', mg._log2)):
                if hasattr(m, a):
                    setattr(m, a, f)
            if hasattr(m, 'get_multiprocessor_count'):
                m.get_multiprocessor_count = lambda *a, **k: 148
    _stub('apex')
    _stub('apex.normalization')
    _stub('apex.normalization.fused_layer_norm', FusedRMSNorm=_FusedRMSNorm)

    class _Registry:
        def register_module(self, *a, **k):
            return lambda cls: cls
    _stub('kairos.apis').__path__ = []
    _stub('kairos.apis.builder', DITS=_Registry())
    _stub('kairos.third_party.fla.layers.gated_deltanet_with_tp', GatedDeltaNet=None)
    _stub('fla').__path__ = []
    _stub('fla.layers', GatedDeltaNet=GatedDeltaNet)
    _stub('fla.utils', autotune_cache_kwargs={})
    dits = ref / 'kairos' / 'modules' / 'dits'
    _stub('kairos.modules.dits').__path__ = [str(dits)]
    torch.compile = lambda *a, **k: (lambda f: f)
    spec = importlib.util.spec_from_file_location('kairos.modules.dits.kairos_dit', dits / 'kairos_dit.py')
    mod = importlib.util.module_from_spec(spec)
    mod.__package__ = 'kairos.modules.dits'
    sys.modules[spec.name] = mod
    spec.loader.exec_module(mod)
    mod.FLASH_ATTN_2_AVAILABLE = False
    mod.FLASH_ATTN_3_AVAILABLE = False
    mod.SAGE_ATTN_AVAILABLE = False
    mod.fla_Cahce = Cache
    return mod, GatedDeltaNet


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--ref', default=os.environ.get('KAIROS_REF', ''))
    args = ap.parse_args()
    if not args.ref:
        raise SystemExit('pass --ref <reference checkout> or set KAIROS_REF')
    kd, GDN = load(Path(args.ref))
    torch.manual_seed(13)
    dim, heads, ffn, eps = 256, 2, 512, 1e-6
    blk = kd.DiTBlock(False, dim, heads, ffn, eps, use_linear_attn=True, gateddeltanet_layer_idx=0,
                      block_idx=0).float().eval()
    blk.gated_delta = GDN(hidden_size=dim, num_heads=heads, head_dim=128, expand_v=1, mode='chunk',
                          use_gate=True, norm_eps=eps, layer_idx=0).float().eval()
    with torch.no_grad():
        for name, p in blk.named_parameters():
            if name == 'modulation' or name.startswith('gated_delta.'):
                continue          # modulation keeps randn / sqrt(dim); the layer its own init
            if name.endswith('norm_q.weight') or name.endswith('norm_k.weight') or name == 'cross_attn_norm.weight':
                p.uniform_(0.5, 1.5)
            else:
                p.normal_(0.0, 0.02 if p.dim() > 1 else 0.05)
        blk.gated_delta.o_norm.weight.uniform_(0.5, 1.5)
    seen = {'x': [], 'o': []}

    def hook(m, inp, out):
        seen['x'].append(inp[0].detach().clone())
        seen['o'].append(out[0].detach().clone())
    blk.gated_delta.register_forward_hook(hook)
    f, h, w = 2, 4, 16
    T = f * h * w                       # 128 tokens: 8 pieces of 16 through the cache
    x = torch.randn(1, T, dim)
    context = torch.randn(1, 16, dim)
    t_mod = torch.randn(1, 6, dim) * 0.1
    freqs = torch.zeros(T, 1, 64, dtype=torch.complex64)   # unused by the GDN branch
    with torch.no_grad():
        y = blk(x.clone(), context, t_mod, freqs, (f, h, w))
    assert len(seen['x']) == 8
    torch.save(dict(state_dict={k: v.clone() for k, v in blk.state_dict().items()}, x=x, context=context,
                    t_mod=t_mod, grid=(f, h, w), dim=dim, heads=heads, head_dim=128, ffn_dim=ffn, eps=eps,
                    gdn_in=torch.cat(seen['x'], 1), gdn_out=torch.cat(seen['o'], 1), pieces=8, out=y), OUT)
    print(f'wrote {OUT} (out std {float(y.std()):.4f}, gdn_out std {float(torch.cat(seen["o"], 1).std()):.4f})')


if __name__ == '__main__':
    main()
