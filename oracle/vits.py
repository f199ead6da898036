"""Oracle for the VITS synthesizer (SynthesizerTrnMs768NSFsid) CPU path.

TEST INFRASTRUCTURE ONLY (see ``oracle/ops.py``).  A numpy restatement of the
reference's numpy-backend inference, ``SynthesizerTrn.infer_controlled``
(``runtime/models/vits.py:2551-2598``) and everything under it, in float32.
``synth(..., taps=d)`` also records the per-layer activations that the CUDA
path is compared against layer by layer.
"""

from __future__ import annotations

import math

import numpy as np

from . import ops

F32 = np.float32


class VitsShape:
    """Architecture derived from the weights + config array.

    Mirrors ``VitsConfig`` (``runtime/models/vits.py:166-249``) for the
    checkpoint format that carries a full config array.
    """

    def __init__(self, w: dict, cfg: list):
        self.hidden = int(w["enc_p.emb_phone.weight"].shape[0])
        self.phone_dim = int(w["enc_p.emb_phone.weight"].shape[1])
        self.filter = int(w["enc_p.encoder.ffn_layers.0.conv_1.weight"].shape[0])
        n = 0
        while f"enc_p.encoder.attn_layers.{n}.conv_q.weight" in w:
            n += 1
        self.n_layers = n
        self.kc = int(w["enc_p.encoder.attn_layers.0.emb_rel_k"].shape[2])
        self.heads = self.hidden // self.kc
        self.rates = [int(r) for r in cfg[12]]
        self.up0 = int(cfg[13])
        self.kernels = [int(k) for k in cfg[14]]
        self.sr = int(cfg[17])
        self.n_ups = len(self.rates)
        self.upp = int(np.prod(self.rates))
        self.noise_strides = []
        for i in range(self.n_ups):
            k = int(w[f"dec.noise_convs.{i}.weight"].shape[2])
            self.noise_strides.append(k // 2 if i < self.n_ups - 1 else 1)
        self.gin = int(w["emb_g.weight"].shape[1])


def rel_embeddings(emb, length, window=10):
    """``_get_relative_embeddings`` (``runtime/models/vits.py:448-462``)."""
    pad = max(length - (window + 1), 0)
    s0 = max((window + 1) - length, 0)
    e = np.pad(emb, ((0, 0), (pad, pad), (0, 0))) if pad > 0 else emb
    return e[:, s0:s0 + 2 * length - 1, :]


def rel_to_abs(x):
    """``[b,h,l,2l-1] -> [b,h,l,l]`` (``runtime/models/vits.py:465-472``)."""
    b, h, L, _ = x.shape
    x = np.pad(x, ((0, 0), (0, 0), (0, 0), (0, 1))).reshape(b, h, L * 2 * L)
    x = np.pad(x, ((0, 0), (0, 0), (0, L - 1))).reshape(b, h, L + 1, 2 * L - 1)
    return x[:, :, :L, L - 1:]


def abs_to_rel(x):
    """``[b,h,l,l] -> [b,h,l,2l-1]`` (``runtime/models/vits.py:475-482``)."""
    b, h, L, _ = x.shape
    x = np.pad(x, ((0, 0), (0, 0), (0, 0), (0, L - 1))).reshape(b, h, L * L + L * (L - 1))
    x = np.pad(x, ((0, 0), (0, 0), (L, 0))).reshape(b, h, L, 2 * L)
    return x[:, :, :, 1:]


def _tap(taps, name, arr):
    if taps is not None:
        taps[name] = np.array(arr, dtype=F32, copy=True)


def text_encoder(w, S: VitsShape, phone, pitch, taps=None):
    """embed + 6 relative-attention layers + proj.

    ``_TextEncoder.embed`` (:499-538), the ``*sqrt(h)`` / leaky 0.1 of
    ``infer_controlled`` (:2569-2571), ``_TextEncoder.encode`` numpy branch
    (:962-1049) and ``stats`` (:1051-1059).  Returns ``m, logs`` ``[1,h,P]``.
    """
    h = S.hidden
    x = ops.linear(phone, w["enc_p.emb_phone.weight"], w["enc_p.emb_phone.bias"])
    x = x + ops.embedding(pitch, w["enc_p.emb_pitch.weight"])
    x = x * math.sqrt(h)
    x = ops.leaky_relu(x, 0.1)
    _tap(taps, "enc.embed", x[0])                   # [P, h]
    x = x.transpose(0, 2, 1)                         # [1, h, P]
    P = x.shape[-1]
    for i in range(S.n_layers):
        p = f"enc_p.encoder.attn_layers.{i}"
        q = ops.conv1d(x, w[p + ".conv_q.weight"], w[p + ".conv_q.bias"])
        k = ops.conv1d(x, w[p + ".conv_k.weight"], w[p + ".conv_k.bias"])
        v = ops.conv1d(x, w[p + ".conv_v.weight"], w[p + ".conv_v.bias"])
        qh = q.reshape(1, S.heads, S.kc, P).transpose(0, 1, 3, 2)
        kh = k.reshape(1, S.heads, S.kc, P).transpose(0, 1, 3, 2)
        vh = v.reshape(1, S.heads, S.kc, P).transpose(0, 1, 3, 2)
        qs = qh / math.sqrt(S.kc)
        scores = np.matmul(qs, np.ascontiguousarray(kh.swapaxes(-1, -2)))
        used_k = rel_embeddings(w[p + ".emb_rel_k"], P)
        scores = scores + rel_to_abs(np.matmul(qs, np.ascontiguousarray(used_k[0].T)))
        pa = ops.softmax(scores)
        out = np.matmul(pa, vh)
        used_v = rel_embeddings(w[p + ".emb_rel_v"], P)
        out = out + np.matmul(abs_to_rel(pa), np.ascontiguousarray(used_v[0]))
        a = out.transpose(0, 1, 3, 2).reshape(1, h, P)
        a = ops.conv1d(a, w[p + ".conv_o.weight"], w[p + ".conv_o.bias"])
        _tap(taps, f"enc.l{i}.attn", a[0].T)
        x = ops.layer_norm((x + a).transpose(0, 2, 1),
                           w[f"enc_p.encoder.norm_layers_1.{i}.gamma"],
                           w[f"enc_p.encoder.norm_layers_1.{i}.beta"]).transpose(0, 2, 1)
        f = f"enc_p.encoder.ffn_layers.{i}"
        y = ops.conv1d(x, w[f + ".conv_1.weight"], w[f + ".conv_1.bias"], padding=1)
        y = ops.relu(y)
        y = ops.conv1d(y, w[f + ".conv_2.weight"], w[f + ".conv_2.bias"], padding=1)
        x = ops.layer_norm((x + y).transpose(0, 2, 1),
                           w[f"enc_p.encoder.norm_layers_2.{i}.gamma"],
                           w[f"enc_p.encoder.norm_layers_2.{i}.beta"]).transpose(0, 2, 1)
        _tap(taps, f"enc.l{i}", x[0].T)               # [P, h]
    st = ops.conv1d(x, w["enc_p.proj.weight"], w["enc_p.proj.bias"])
    m, logs = st[:, :h, :], st[:, h:, :]
    _tap(taps, "enc.m", m[0].T)
    _tap(taps, "enc.logs", logs[0].T)
    return m, logs


def flow_reverse(w, S: VitsShape, z, g):
    """``_FlowBlock.reverse`` (:1255-1268) with ``_rc_reverse`` (:1086-1098)
    and the numpy ``_wn`` (:1100-1145); x_mask is all ones at inference."""
    h = S.hidden
    half = h // 2
    for idx in (6, 4, 2, 0):
        z = np.flip(z, axis=1)
        p = f"flow.flows.{idx}"
        x0, x1 = z[:, :half, :], z[:, half:, :]
        hh = ops.conv1d(x0, w[p + ".pre.weight"], w[p + ".pre.bias"])
        gc = ops.conv1d(g, ops.deweight_norm(w[p + ".enc.cond_layer.weight_v"],
                                             w[p + ".enc.cond_layer.weight_g"]),
                        w[p + ".enc.cond_layer.bias"])
        acc = np.zeros_like(hh)
        for i in range(3):
            xin = ops.conv1d(hh, ops.deweight_norm(w[p + f".enc.in_layers.{i}.weight_v"],
                                                   w[p + f".enc.in_layers.{i}.weight_g"]),
                             w[p + f".enc.in_layers.{i}.bias"], padding=2)
            gl = gc[:, i * 2 * h:(i + 1) * 2 * h, :]
            t = xin + gl
            acts = np.tanh(t)[:, :h, :] * ops.sigmoid(t[:, h:, :])
            rs = ops.conv1d(acts, ops.deweight_norm(w[p + f".enc.res_skip_layers.{i}.weight_v"],
                                                    w[p + f".enc.res_skip_layers.{i}.weight_g"]),
                            w[p + f".enc.res_skip_layers.{i}.bias"])
            if i < 2:
                hh = hh + rs[:, :h, :]
                acc = acc + rs[:, h:, :]
            else:
                acc = acc + rs
        m = ops.conv1d(acc, w[p + ".post.weight"], w[p + ".post.bias"])
        z = np.concatenate([x0, x1 - m], axis=1)
    return z


def phase_offsets(S: VitsShape, f0):
    """Full-length per-frame phase carry ``fmod(cumsum(...))`` (``runtime/models/vits.py:2396-2407``)."""
    f0r = f0[:, None].transpose(0, 2, 1)
    rad = f0r / S.sr * np.arange(1, S.upp + 1, dtype=F32)[None, None, :]
    rad2 = np.fmod(rad[..., -1:] + 0.5, 1.0) - 0.5
    return np.fmod(np.cumsum(rad2, axis=1), 1.0)


def sine_source(w, S: VitsShape, f0, ns, off=None):
    """SineGen (harmonic_num 0) + SourceModuleHnNSF, full-length phase path.

    ``_GeneratorNSF._sine_gen`` (:1468-1501): per-frame phase ramp
    ``f0/sr*[1..upp]``, fmod-cumsum phase carry between frames, 0.1*sin(2 pi .),
    uv gate, noise amplitude 0.003 voiced / 0.1/3 unvoiced, 1x1 linear, tanh.
    Returns ``har [1,1,P*upp]``.
    """
    upp, sr = S.upp, S.sr
    f0r = f0[:, None].transpose(0, 2, 1)                     # [1,P,1]
    rad = f0r / sr * np.arange(1, upp + 1, dtype=F32)[None, None, :]
    if off is None:
        rad2 = np.fmod(rad[..., -1:] + 0.5, 1.0) - 0.5
        acc = np.fmod(np.cumsum(rad2, axis=1), 1.0)
        rad = rad.copy()
        rad[:, 1:, :] += acc[:, :-1, :]
    else:  # segment with per-frame total phase offsets (:1490-1491)
        rad = rad + np.asarray(off, dtype=F32)
    rad = rad.reshape(1, -1, 1)
    sine = np.sin(2 * np.pi * rad) * 0.1
    uv = np.repeat((f0r > 0).astype(F32), upp, axis=1)
    amp = uv * 0.003 + (1 - uv) * 0.1 / 3
    sine = sine * uv + amp * ns
    lin = ops.linear(sine, w["dec.m_source.l_linear.weight"], w["dec.m_source.l_linear.bias"])
    return np.tanh(lin).transpose(0, 2, 1)


def _resblock(w, base, x, k):
    """``_ResBlock1.forward`` (:1285-1311)."""
    for j, d in enumerate((1, 3, 5)):
        c = ops.leaky_relu(x, 0.1)
        c = ops.conv1d(c, ops.deweight_norm(w[f"{base}.convs1.{j}.weight_v"],
                                            w[f"{base}.convs1.{j}.weight_g"]),
                       w[f"{base}.convs1.{j}.bias"], dilation=d, padding=(k * d - d) // 2)
        c = ops.leaky_relu(c, 0.1)
        c = ops.conv1d(c, ops.deweight_norm(w[f"{base}.convs2.{j}.weight_v"],
                                            w[f"{base}.convs2.{j}.weight_g"]),
                       w[f"{base}.convs2.{j}.bias"], padding=(k - 1) // 2)
        x = c + x
    return x


def generator(w, S: VitsShape, z, f0, g, ns, taps=None, off=None):
    """``_GeneratorNSF.forward`` numpy branch (:2133-2231) and the per-stage
    ``_dec_ups_single`` (:1616-1636).  Returns the waveform ``[1,1,P*upp]``."""
    har = sine_source(w, S, f0, ns, off)
    _tap(taps, "dec.har", har[0, 0])
    x = ops.conv1d(z, w["dec.conv_pre.weight"], w["dec.conv_pre.bias"], padding=3)
    x = x + ops.conv1d(g, w["dec.cond.weight"], w["dec.cond.bias"])
    _tap(taps, "dec.pre", x[0].T)
    for i in range(S.n_ups):
        x = ops.leaky_relu(x, 0.1)
        wu = ops.deweight_norm(w[f"dec.ups.{i}.weight_v"], w[f"dec.ups.{i}.weight_g"])
        x = ops.conv_transpose1d(x, wu, w[f"dec.ups.{i}.bias"], stride=S.rates[i],
                                 padding=(S.kernels[i] - S.rates[i]) // 2)
        s = S.noise_strides[i]
        x = x + ops.conv1d(har, w[f"dec.noise_convs.{i}.weight"],
                           w[f"dec.noise_convs.{i}.bias"], stride=s, padding=s // 2)
        _tap(taps, f"dec.s{i}.ups", x[0].T)
        xs = None
        for j, k in enumerate((3, 7, 11)):
            o = _resblock(w, f"dec.resblocks.{i * 3 + j}", x, k)
            xs = o if xs is None else xs + o
        x = xs / 3
        _tap(taps, f"dec.s{i}.out", x[0].T)
    x = ops.leaky_relu(x, 0.01)
    x = ops.conv1d(x, w["dec.conv_post.weight"], None, padding=3)
    _tap(taps, "dec.post", x[0, 0])
    return np.tanh(x)


def synth(w, cfg, phone, pitch, nsff0, sid, nz, ns, taps=None):
    """``SynthesizerTrn.infer_controlled`` (:2551-2598): waveform ``[1,1,P*upp]``."""
    S = VitsShape(w, cfg)
    g = ops.embedding(sid, w["emb_g.weight"])[0].reshape(1, -1, 1)
    m, logs = text_encoder(w, S, phone, pitch, taps)
    z_p = m + np.exp(logs) * nz * 0.66666
    _tap(taps, "enc.zp", z_p[0].T)
    z = flow_reverse(w, S, z_p, g)
    _tap(taps, "flow.z", z[0].T)
    return generator(w, S, z, nsff0, g, ns, taps)


FLOW_PAD, DEC_PAD = 24, 16  # runtime/models/vits.py:148-152


def synth_partial(w, cfg, phone, pitch, nsff0, sid, nz, ns, head, length):
    """``SynthesizerTrn._infer_partial`` (:2539-2548) with ``_partial_prep``
    (:2422-2476): full text encoder, flow from ``max(head-24-16, 0)``, generator
    on frames ``[max(head-16,0), min(P, head+length+16))`` with phase offsets,
    output samples of frames ``[head, head+length)``."""
    S = VitsShape(w, cfg)
    P = phone.shape[1]
    upp = S.upp
    g = ops.embedding(sid, w["emb_g.weight"])[0].reshape(1, -1, 1)
    m, logs = text_encoder(w, S, phone, pitch)
    fh = max(head - FLOW_PAD - DEC_PAD, 0)
    z_p = m[:, :, fh:] + np.exp(logs[:, :, fh:]) * nz[:, :, fh:] * 0.66666
    z = flow_reverse(w, S, z_p, g)
    zs, ze = max(head - DEC_PAD, 0), min(P, head + length + DEC_PAD)
    z_seg = z[:, :, zs - fh:ze - fh]
    acc = phase_offsets(S, nsff0)
    n = ze - zs
    if zs == 0:
        off = np.zeros((1, n, 1), dtype=F32)
        if n > 1:
            off[:, 1:, :] = acc[:, :n - 1, :]
    else:
        off = acc[:, zs - 1:zs - 1 + n, :]
    o = generator(w, S, z_seg, nsff0[:, zs:ze], g, ns[:, zs * upp:ze * upp, :], off=off)
    s0 = (head - zs) * upp
    return o[:, :, s0:s0 + length * upp]
