"""Oracle for the HuBERT-base encoder CPU path.

TEST INFRASTRUCTURE ONLY (see ``oracle/ops.py``).  A numpy restatement of the
reference's numpy-backend ``HubertEncoder.encode(x, version=2)``
(``runtime/models/hubert.py:564-589``): conv feature extractor, feature
projection, grouped positional conv, 12 post-LN transformer layers.
"""

from __future__ import annotations

import numpy as np

from . import ops

F32 = np.float32


def prepare(sd: dict) -> dict:
    """Fold the positional conv's weight norm (dim=2) like
    ``HubertEncoder._load_and_prepare`` (``runtime/models/hubert.py:499-559``):
    ``W = g * v / ||v||`` with the norm over axes (0, 1), in float64 then f32."""
    sd = {k: np.asarray(v, dtype=F32) for k, v in sd.items()}
    g = sd["encoder.pos_conv_embed.conv.weight_g"]
    v = sd["encoder.pos_conv_embed.conv.weight_v"]
    norm = np.sqrt(np.sum(v.astype(np.float64) ** 2, axis=(0, 1), keepdims=True))
    sd["_pos_conv_weight"] = (g * (v / norm.astype(F32))).astype(F32)
    return sd


def _tap(taps, name, arr):
    if taps is not None:
        taps[name] = np.array(arr, dtype=F32, copy=True)


def grouped_conv1d(x, w, b, groups, padding):
    """Per-group conv1d then concat (``runtime/models/hubert.py:301-337``)."""
    C = x.shape[1]
    cpg = C // groups
    opg = w.shape[0] // groups
    parts = [ops.conv1d(x[:, g * cpg:(g + 1) * cpg], w[g * opg:(g + 1) * opg],
                        b[g * opg:(g + 1) * opg], padding=padding)
             for g in range(groups)]
    return np.concatenate(parts, axis=1)


def encode(sd: dict, x: np.ndarray, taps=None, version: int = 2) -> np.ndarray:
    """``[1,T]`` 16 kHz waveform -> ``[1,L,768]`` last hidden state (version 2),
    or layer 9's output through ``final_proj`` ``[1,L,256]`` (version 1,
    ``runtime/models/hubert.py:580-586``)."""
    x = np.asarray(x, dtype=F32)
    h = x[:, None, :]
    for i in range(7):
        wc = sd[f"feature_extractor.conv_layers.{i}.conv.weight"]
        h = ops.conv1d(h, wc, None, stride=5 if i == 0 else 2)     # :658-705
        if i == 0:
            h = ops.group_norm(h, sd["feature_extractor.conv_layers.0.layer_norm.weight"],
                               sd["feature_extractor.conv_layers.0.layer_norm.bias"], 512)
        h = ops.gelu_erf(h)
        _tap(taps, f"conv{i}", h[0].T)
    h = h.transpose(0, 2, 1)                                         # [1, L, 512]
    h = ops.layer_norm(h, sd["feature_projection.layer_norm.weight"],
                       sd["feature_projection.layer_norm.bias"])      # :775-806
    h = ops.linear(h, sd["feature_projection.projection.weight"], None)
    h = h + sd["feature_projection.projection.bias"].reshape(1, -1)
    _tap(taps, "proj", h[0])
    L = h.shape[1]
    pos = grouped_conv1d(h.transpose(0, 2, 1), sd["_pos_conv_weight"],
                         sd["encoder.pos_conv_embed.conv.bias"], 16, 64)[:, :, :L]
    pos = ops.gelu_erf(pos).transpose(0, 2, 1)                     # :838-866
    _tap(taps, "pos", pos[0])
    h = ops.layer_norm(h + pos, sd["encoder.layer_norm.weight"], sd["encoder.layer_norm.bias"])
    scale = 64.0 ** -0.5
    for i in range(9 if version == 1 else 12):                       # :1262-1287
        p = f"encoder.layers.{i}."
        q = ops.linear(h, sd[p + "attention.q_proj.weight"], sd[p + "attention.q_proj.bias"]) * scale
        k = ops.linear(h, sd[p + "attention.k_proj.weight"], sd[p + "attention.k_proj.bias"])
        v = ops.linear(h, sd[p + "attention.v_proj.weight"], sd[p + "attention.v_proj.bias"])
        B, T, C = q.shape
        qh = q.reshape(B, T, 12, 64).transpose(0, 2, 1, 3)
        kh = k.reshape(B, T, 12, 64).transpose(0, 2, 1, 3)
        vh = v.reshape(B, T, 12, 64).transpose(0, 2, 1, 3)
        att = ops.softmax(np.matmul(qh, np.ascontiguousarray(kh.swapaxes(-1, -2))))
        ctx = np.matmul(att, np.ascontiguousarray(vh)).transpose(0, 2, 1, 3).reshape(B, T, C)
        a = ops.linear(ctx, sd[p + "attention.out_proj.weight"], sd[p + "attention.out_proj.bias"])
        h = ops.layer_norm(h + a, sd[p + "layer_norm.weight"], sd[p + "layer_norm.bias"])
        f = ops.linear(h, sd[p + "feed_forward.intermediate_dense.weight"],
                       sd[p + "feed_forward.intermediate_dense.bias"])
        f = ops.linear(ops.gelu_erf(f), sd[p + "feed_forward.output_dense.weight"],
                       sd[p + "feed_forward.output_dense.bias"])
        h = ops.layer_norm(h + f, sd[p + "final_layer_norm.weight"], sd[p + "final_layer_norm.bias"])
        _tap(taps, f"layer{i}", h[0])
    if version == 1:
        return ops.linear(h, sd["final_proj.weight"], sd["final_proj.bias"])
    return h
