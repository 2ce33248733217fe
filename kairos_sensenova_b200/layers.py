"""``GatedDeltaNet`` layer drop-in (chunk mode) on the sm_100a kernels.

Constructor arguments, parameter names/shapes (so reference state dicts load
unchanged: ``q_proj, k_proj, v_proj, a_proj, b_proj, g_proj, o_proj, A_log,
dt_bias, {q,k,v}_conv1d.weight, o_norm.weight``) and the forward signature
follow ``kairos/third_party/fla/layers/gated_deltanet.py:88-319``:
``forward(hidden_states, attention_mask=None, past_key_values=None,
use_cache=False, output_attentions=False, **kwargs) -> (o, None, past_key_values)``.

Projections are plain cuBLAS GEMMs (``nn.Linear``); the short convolutions,
SiLU and gates run in one prologue kernel, the recurrence in the chunked GDN
kernels and the gated RMSNorm in one epilogue kernel.  Recurrent caches work
as in the reference (``gated_deltanet.py:225-253,273-305``): with
``past_key_values`` the layer reads this layer's conv states (the last W raw
q/k/v projection inputs) and recurrent state, continues the sequence from them,
and with ``use_cache`` stores the new ones -- so a long sequence walked in
pieces through one :class:`Cache` gives the one-shot result (the DiT block's
GDN loop, ``kairos_dit.py:880-922``).  Padding masks (``attention_mask``) are
not implemented and raise ``NotImplementedError``.  The reference routes
``q_len <= 64`` to its fused-recurrent kernel (``gated_deltanet.py:220``);
the chunk kernels here are exact for every length, so they serve all lengths.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn

from .fused_ops import gdn_prologue, rms_norm_gated
from .gated_delta_rule import chunk_gated_delta_rule


class Cache:
    """Per-layer recurrent-state cache with the interface ``GatedDeltaNet`` uses
    (``fla/models/utils.py:283-382``, ``FLACache``): ``len(cache)`` is the number of
    layers that stored state, ``cache[i]`` that layer's dict (``recurrent_state``,
    ``attn_state``, ``conv_state``, ``ffn_state``), ``update(..., layer_idx,
    offset)`` stores new states (growing the layer list to ``layer_idx``) and counts
    the tokens seen by layer 0."""

    def __init__(self, seen_tokens: int = 0):
        self.layers = []
        self._seen_tokens = int(seen_tokens)

    @classmethod
    def from_legacy_cache(cls, past_key_values=None, seen_tokens: int = 0):
        cache = cls(seen_tokens)
        if isinstance(past_key_values, (list, tuple)):
            cache.layers = [dict(st) for st in past_key_values]
        return cache

    def to_legacy_cache(self):
        return tuple(self.layers)

    def __len__(self):
        return len(self.layers)

    def __getitem__(self, layer_idx):
        if layer_idx >= len(self.layers):
            raise KeyError(f"Cache only have {len(self.layers)} layers, however accessed {layer_idx} out of bounds")
        return self.layers[layer_idx]

    def __iter__(self):
        yield from self.layers

    def update(self, recurrent_state=None, attn_state=None, conv_state=None, ffn_state=None, layer_idx=0,
               offset=1, cache_kwargs=None):
        while len(self.layers) <= layer_idx:
            self.layers.append(dict(recurrent_state=None, attn_state=None, conv_state=None, ffn_state=None))
        if layer_idx == 0:
            self._seen_tokens += int(offset)
        st = self.layers[layer_idx]
        if recurrent_state is not None:
            st['recurrent_state'] = recurrent_state
        if attn_state is not None:
            old = st['attn_state']
            st['attn_state'] = tuple(attn_state) if old is None else tuple(
                torch.cat([a, b], 1) for a, b in zip(old, attn_state))
        if conv_state is not None:
            st['conv_state'] = conv_state
        if ffn_state is not None:
            st['ffn_state'] = ffn_state
        return st

    def get_seq_length(self, layer_idx=0):
        return self._seen_tokens if len(self.layers) > (layer_idx or 0) else 0


def _next_conv_state(prev, x, W):
    """The conv state after the piece ``x [B, T, C]``: the last W inputs of the
    sequence so far, ``[B, C, W]`` (older ones from ``prev`` when T < W), as
    ``causal_conv1d_states_fwd_kernel`` forms it (``fla/modules/convolution.py:534-577``)."""
    B, T, C = x.shape
    xt = x.transpose(1, 2)
    if T >= W:
        return xt[..., T - W:].contiguous()
    if prev is None:
        prev = x.new_zeros(B, C, W)
    return torch.cat([prev.to(x.dtype), xt], -1)[..., -W:].contiguous()


class ShortConvolution(nn.Conv1d):
    """Parameter holder with the reference's layout (depthwise ``nn.Conv1d``,
    weight ``[C, 1, W]``; ``fla/modules/convolution.py:801-853``)."""

    def __init__(self, hidden_size, kernel_size, bias=False, activation='silu', **kwargs):
        super().__init__(hidden_size, hidden_size, kernel_size, groups=hidden_size, bias=bias,
                         padding=kernel_size - 1)
        self.hidden_size = hidden_size
        self.activation = activation


class FusedRMSNormGated(nn.Module):
    """Parameter holder + forward of ``FusedRMSNormGated`` (swish gate)."""

    def __init__(self, hidden_size, elementwise_affine=True, eps=1e-5, activation='swish'):
        super().__init__()
        if activation not in ('swish', 'silu'):
            raise ValueError(f'Unsupported activation: {activation}')
        self.hidden_size, self.eps, self.activation = hidden_size, eps, activation
        self.weight = nn.Parameter(torch.ones(hidden_size))

    def forward(self, x, g, residual=None, prenorm=False, residual_in_fp32=False, tp_group=None):
        if residual is not None or prenorm:
            raise NotImplementedError('residual/prenorm variants are not on this path')
        return rms_norm_gated(x, g, self.weight, self.eps)


class GatedDeltaNet(nn.Module):
    def __init__(self, hidden_size=2048, expand_v=2, head_dim=256, num_heads=6, num_v_heads=None,
                 mode='chunk', use_gate=True, use_short_conv=True, allow_neg_eigval=False,
                 conv_size=4, conv_bias=False, layer_idx=None, norm_eps=1e-5, **kwargs):
        super().__init__()
        self.mode = mode
        self.allow_neg_eigval = allow_neg_eigval
        self.hidden_size = hidden_size
        self.expand_v = expand_v
        self.use_gate = use_gate
        self.use_short_conv = use_short_conv
        self.conv_size = conv_size
        self.conv_bias = conv_bias
        self.head_dim = head_dim
        self.num_heads = num_heads
        self.num_v_heads = num_v_heads if num_v_heads is not None else num_heads
        self.head_k_dim = head_dim
        self.head_v_dim = int(head_dim * expand_v)
        self.key_dim = int(self.num_heads * self.head_k_dim)
        self.value_dim = int(self.num_v_heads * self.head_v_dim)
        self.layer_idx = layer_idx
        if not math.isclose(self.num_v_heads * head_dim * expand_v, self.value_dim, rel_tol=1e-5):
            raise ValueError(f"expand_v={expand_v} does not produce an integer value_dim")
        if self.num_v_heads != self.num_heads:
            raise NotImplementedError('num_v_heads != num_heads (GVA) is not on this path')
        if not (use_gate and use_short_conv):
            raise NotImplementedError('use_gate=False / use_short_conv=False are not on this path')
        assert mode in ['chunk', 'fused_recurrent'], f"Not supported mode `{mode}`."
        self.q_proj = nn.Linear(hidden_size, self.key_dim, bias=False)
        self.k_proj = nn.Linear(hidden_size, self.key_dim, bias=False)
        self.v_proj = nn.Linear(hidden_size, self.value_dim, bias=False)
        self.a_proj = nn.Linear(hidden_size, self.num_v_heads, bias=False)
        self.b_proj = nn.Linear(hidden_size, self.num_v_heads, bias=False)
        A = torch.empty(self.num_v_heads, dtype=torch.float32).uniform_(0, 16)
        self.A_log = nn.Parameter(torch.log(A))
        dt_min, dt_max, dt_init_floor = 0.001, 0.1, 1e-4
        dt = torch.exp(torch.rand(self.num_v_heads) * (math.log(dt_max) - math.log(dt_min)) + math.log(dt_min))
        dt = torch.clamp(dt, min=dt_init_floor)
        self.dt_bias = nn.Parameter(dt + torch.log(-torch.expm1(-dt)))
        self.q_conv1d = ShortConvolution(self.key_dim, conv_size, bias=conv_bias)
        self.k_conv1d = ShortConvolution(self.key_dim, conv_size, bias=conv_bias)
        self.v_conv1d = ShortConvolution(self.value_dim, conv_size, bias=conv_bias)
        self.g_proj = nn.Linear(hidden_size, self.value_dim, bias=False)
        self.o_norm = FusedRMSNormGated(self.head_v_dim, eps=norm_eps)
        self.o_proj = nn.Linear(self.value_dim, hidden_size, bias=False)

    def forward(self, hidden_states, attention_mask=None, past_key_values=None, use_cache=False,
                output_attentions=False, **kwargs):
        if attention_mask is not None:
            raise NotImplementedError('padding masks are not implemented on this path')
        B, T, _ = hidden_states.shape
        H = self.num_heads
        cu_seqlens = kwargs.get('cu_seqlens')
        last_state = None
        layer_idx = self.layer_idx or 0
        if past_key_values is not None and len(past_key_values) > layer_idx:
            last_state = past_key_values[layer_idx]
        if last_state is not None and cu_seqlens is not None:
            raise NotImplementedError('a conv cache together with cu_seqlens is not on this path')
        conv_prev = last_state['conv_state'] if last_state is not None else None
        x2 = hidden_states.reshape(B * T, -1)
        xq, xk, xv = self.q_proj(x2), self.k_proj(x2), self.v_proj(x2)
        cb = lambda c: None if c.bias is None else c.bias  # noqa: E731
        q, k, v, g, beta = gdn_prologue(
            xq, xk, xv, self.a_proj(x2), self.b_proj(x2),
            self.q_conv1d.weight[:, 0], self.k_conv1d.weight[:, 0], self.v_conv1d.weight[:, 0],
            self.A_log, self.dt_bias, H, B, T, cb(self.q_conv1d), cb(self.k_conv1d), cb(self.v_conv1d),
            self.allow_neg_eigval, conv_cache=conv_prev)
        recurrent_state = last_state['recurrent_state'] if last_state is not None else None
        o, recurrent_state = chunk_gated_delta_rule(q, k, v, g, beta, initial_state=recurrent_state,
                                                    output_final_state=use_cache, cu_seqlens=cu_seqlens,
                                                    use_qk_l2norm_in_kernel=True)
        if past_key_values is not None:
            # as the reference: the conv states are only formed with use_cache
            prev = conv_prev if conv_prev is not None else (None, None, None)
            conv_state = tuple(_next_conv_state(p, x.reshape(B, T, -1), self.conv_size) if use_cache else None
                               for p, x in zip(prev, (xq, xk, xv)))
            past_key_values.update(recurrent_state=recurrent_state, conv_state=conv_state,
                                   layer_idx=layer_idx, offset=T)
        gate = self.g_proj(x2).reshape(B, T, H, self.head_v_dim)
        o = self.o_norm(o, gate)
        o = self.o_proj(o.reshape(B, T, self.value_dim).to(hidden_states.dtype))
        return o, None, past_key_values
