"""Decode steps of standard attention modules run on the compressed archive.

Same entry points as flashcodec/patch_attention.py:105-151
(``apply_codec_attention``, ``remove_codec_attention``,
``codec_attention_stats``).  The patched forward keeps the model's own
projections, QK-norm and rotary embedding, appends the new key/value token to
the layer's codec streams and computes attention with one
``codec_decode_attention`` launch (fc_decode_attn): the (S, D) view is never
reconstructed during decode.

The rotary embedding and the append run as one fc_rope_kv_append launch
once the model's rotary function has been checked, on its first decode step,
to give bit-identical results to the fused kernel (``_fused_rope``); the
reference runs them as separate torch ops and appends
(flashcodec/patch_attention.py:82-94).

Taken when (anything else runs the original forward, silently, as in
flashcodec/patch_attention.py:51-63):

* the cache layer is a ``FlashCodecLayer``, the module is in eval mode, the
  step has one query token, ``position_embeddings`` is given, the module has
  no sliding window and its model file defines ``apply_rotary_pos_emb``;
* any batch size.  The reference stops at batch 1
  (flashcodec/patch_attention.py:54).  Without padding transformers passes no
  mask.  A padded batch's mask, a (B, 1, 1, S+1) boolean or additive tensor at
  a decode step, becomes the kernel's per-key visibility
  (fc_decode_attn_masked).  A mask of any other shape keeps the original
  forward.
"""

from __future__ import annotations

import importlib

import torch

from . import _kernels as K
from .cache import append_rotary

_ROPE = {}
_ROPE_EXACT = {}       # (rotary function, dtype) -> the fused kernel matches it bitwise


def _rope_fn(module):
    """``apply_rotary_pos_emb`` of the file that defines the module's class,
    or None."""
    name = type(module).__module__
    fn = _ROPE.get(name)
    if fn is None:
        try:
            fn = getattr(importlib.import_module(name), "apply_rotary_pos_emb", None)
        except Exception:
            fn = None
        _ROPE[name] = fn or False
    return fn or None


def _fused_rope(rope, q, k, v, cos, sin, key_stream):
    """Whether this step's rotary embedding and append may run as one
    fc_rope_kv_append launch.  The first time a model's rotary function is
    seen, the kernel's rotation is compared bitwise with the function's
    output on that step's q and k (the step itself then takes the unfused
    path); functions that differ (partial rotary, interleaved pairs, another
    rounding) keep the unfused path for good."""
    D = q.shape[-1]
    if not (q.dtype == k.dtype == v.dtype == cos.dtype == sin.dtype
            and q.dtype in (torch.float32, torch.bfloat16, torch.float16)
            and (key_stream.dtype is None or key_stream.dtype == k.dtype)
            and D % 2 == 0 and cos.shape == sin.shape and cos.shape[-1] == D
            and cos.numel() // D in (1, q.shape[0])):
        return False
    key = (rope, q.dtype)
    ok = _ROPE_EXACT.get(key)
    if ok is None:
        q_ref, k_ref = rope(q, k, cos, sin)
        q_f, k_f = torch.empty_like(q_ref), torch.empty_like(k_ref)
        K.rope_kv_append(q, k, None, cos, sin, q_f, k_f)
        ok = bool(torch.equal(q_f, q_ref) and torch.equal(k_f, k_ref))
        _ROPE_EXACT[key] = ok
        return False
    return ok


def _key_visibility(attention_mask, batch, keys):
    """(B, keys) visibility from a decode step's attention mask, or None when
    the mask has another form."""
    m = attention_mask
    if m is None or m.dim() != 4 or m.shape[0] != batch or m.shape[-2] != 1 \
            or m.shape[-1] < keys or m.shape[1] != 1:
        return None
    row = m[:, 0, -1, :keys]
    if row.dtype == torch.bool:
        return row
    if row.is_floating_point():          # additive mask: 0 where visible
        return row > torch.finfo(row.dtype).min / 2
    return None


def _codec_layer(module, past_key_values):
    from .hf_cache import FlashCodecLayer
    layers = getattr(past_key_values, "layers", None)
    if layers is None:
        return None
    try:
        layer = layers[module.layer_idx]
    except (IndexError, TypeError):
        return None
    return layer if isinstance(layer, FlashCodecLayer) else None


def _decode_forward(module, orig, hidden_states, position_embeddings=None,
                    attention_mask=None, past_key_values=None, **kwargs):
    layer = _codec_layer(module, past_key_values)
    batch, q_len = hidden_states.shape[0], hidden_states.shape[-2]
    rope = _rope_fn(module)
    visible = None
    if layer is not None and batch != 1 and attention_mask is not None:
        visible = _key_visibility(attention_mask, batch, layer._key_stream.seq_len + 1)
    if (layer is None or module.training or q_len != 1 or position_embeddings is None
            or getattr(module, "sliding_window", None) is not None or rope is None
            or (batch != 1 and attention_mask is not None and visible is None)):
        return orig(hidden_states, position_embeddings=position_embeddings,
                    attention_mask=attention_mask, past_key_values=past_key_values,
                    **kwargs)

    lead = hidden_states.shape[:-1]
    hd = module.head_dim
    q = module.q_proj(hidden_states)
    gate = None
    if module.q_proj.out_features == 2 * module.o_proj.in_features:
        # gated query projection (Qwen3.5 layout): per head [query | gate]
        q, gate = q.view(*lead, -1, 2 * hd).chunk(2, dim=-1)
        gate = gate.reshape(*lead, -1)
    q = q.reshape(*lead, -1, hd)
    k = module.k_proj(hidden_states).view(*lead, -1, hd)
    v = module.v_proj(hidden_states).view(*lead, -1, hd).transpose(1, 2)
    if hasattr(module, "q_norm"):          # QK-norm over (heads, head_dim)
        q = module.q_norm(q)
    if hasattr(module, "k_norm"):
        k = module.k_norm(k)
    cos, sin = position_embeddings
    q, k = q.transpose(1, 2), k.transpose(1, 2)

    if not layer.is_initialized:
        layer.lazy_initialization(k, v)
    ks, vs = layer._key_stream, layer._value_stream
    for st in (ks, vs):                     # prefill's view is not needed now
        if st._rec is not None:
            st.discard_view()
    layer.keys = layer.values = None
    if _fused_rope(rope, q, k, v, cos, sin, ks):
        q = append_rotary(ks, vs, q, k, v, cos, sin)
    else:
        q, k = rope(q, k, cos, sin)
        ks.append(k)
        vs.append(v)
    from .attention import codec_decode_attention
    out = codec_decode_attention(q, ks, vs, scale=module.scaling, visible=visible)
    out = out.transpose(1, 2).reshape(*lead, -1)
    if gate is not None:
        out = out * torch.sigmoid(gate)
    return module.o_proj(out), None


def _supported(module):
    need = ("q_proj", "k_proj", "v_proj", "o_proj", "layer_idx", "head_dim")
    if not all(hasattr(module, a) for a in need):
        return False
    width = module.o_proj.in_features
    return (module.head_dim > 0 and width % module.head_dim == 0
            and module.q_proj.out_features in (width, 2 * width))


def apply_codec_attention(model):
    """Wrap the forward of every supported attention module.  Idempotent;
    returns the number of wrapped modules."""
    n = 0
    for module in model.modules():
        if not _supported(module):
            continue
        n += 1
        if getattr(module, "_flashcodec_orig_forward", None) is not None:
            continue
        orig = module.forward

        def forward(*args, _module=module, _orig=orig, **kw):
            return _decode_forward(_module, _orig, *args, **kw)

        module._flashcodec_orig_forward = orig
        module.forward = forward
    return n


def remove_codec_attention(model):
    """Restore the original forwards; returns how many were restored."""
    n = 0
    for module in model.modules():
        orig = getattr(module, "_flashcodec_orig_forward", None)
        if orig is not None:
            module.forward = orig
            del module._flashcodec_orig_forward
            n += 1
    return n


def codec_attention_stats(model):
    """Number of attention modules currently wrapped."""
    return sum(1 for m in model.modules()
               if getattr(m, "_flashcodec_orig_forward", None) is not None)


__all__ = ["apply_codec_attention", "remove_codec_attention", "codec_attention_stats"]
