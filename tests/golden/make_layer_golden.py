"""Golden fixture for the GatedDeltaNet layer (prologue + chunk op + gated
RMSNorm epilogue), produced by the REFERENCE'S OWN vendored layer
``kairos/third_party/fla/layers/gated_deltanet.py`` on CPU in fp32.

Run in a container where the reference tree is mounted (``--ref`` or
``KAIROS_REF``); the GPU box only reads the committed fixture.  The Triton
kernels of the layer (short convolution, chunk op, fused gated norm) run under
``TRITON_INTERPRET=1`` with the shims of ``make_golden.py`` plus one more: the
SM-count query the convolution uses to pick a tile size
(``fla/utils.py:363``) returns 148, as there is no GPU driver to ask.
"""
from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

os.environ['TRITON_INTERPRET'] = '1'   # must precede the first triton import

import torch  # noqa: E402

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import make_golden as mg  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--ref', default=os.environ.get('KAIROS_REF', ''))
    args = ap.parse_args()
    ref = Path(args.ref)
    assert (ref / 'kairos').is_dir(), 'pass --ref <reference tree>'
    mg.load_triton_chunk(ref)
    from kairos.third_party.fla.layers.gated_deltanet import GatedDeltaNet
    for name, m in list(sys.modules.items()):
        if name.startswith('kairos.third_party.fla') and m is not None:
            for a, f in (('exp', mg._exp), ('exp2', mg._exp2), ('log', mg._log), ('log2', mg._log2)):
                if hasattr(m, a):
                    setattr(m, a, f)
            if hasattr(m, 'get_multiprocessor_count'):
                m.get_multiprocessor_count = lambda *a, **k: 148
    torch.manual_seed(21)
    hidden, H, hd, T = 256, 2, 128, 130
    layer = GatedDeltaNet(hidden_size=hidden, expand_v=1, head_dim=hd, num_heads=H, mode='chunk', use_gate=True,
                          use_short_conv=True, norm_eps=1e-5, layer_idx=0).float().eval()
    with torch.no_grad():
        layer.o_norm.weight.uniform_(0.5, 1.5)
    x = torch.randn(1, T, hidden)
    with torch.no_grad():
        o, _, _ = layer(x)
    torch.save(dict(state_dict={k: v.clone() for k, v in layer.state_dict().items()}, x=x, out=o,
                    hidden=hidden, heads=H, head_dim=hd, norm_eps=1e-5), HERE / 'layer_gdn.pt')
    print(f'wrote layer_gdn.pt (out std {float(o.std()):.4f})')


if __name__ == '__main__':
    main()
