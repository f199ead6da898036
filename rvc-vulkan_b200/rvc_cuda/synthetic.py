"""Seeded synthetic checkpoints and inputs for the RVC inference hot path.

No checkpoints can be downloaded on the machines this library is measured on,
so every test and benchmark builds random-init weights of the real
architectures with the reference's own state-dict key names, and synthetic
inputs with the shapes and value distributions of the measured configs.

Everything is drawn from ``numpy.random.RandomState`` (the frozen legacy
stream), so a seed gives the same arrays on every numpy version and every
machine: golden fixtures store only seeds, outputs and checksums.

Weight distribution: plain weights and biases are N(0, 0.02), LayerNorm
gamma=1 / beta=0 (BASELINE config text "random-init fp32 weights N(0,0.02)").
The checkpoints of the reference use ``torch.nn.utils.weight_norm`` for the
flow and decoder convolutions (``runtime/models/vits.py:416-442``).  For those
``weight_v`` is N(0, 0.02) and ``weight_g`` is set so that the folded weight
W = g * v / ||v|| keeps activations of order one through the stack (a gain per
layer, jittered by 10 %); with g also N(0, 0.02) the decoder would shrink its
signal by ~1e-6 and the waveform test would be vacuous.
"""

from __future__ import annotations

import math

import numpy as np

__all__ = [
    "VITS_V2_40K", "VITS_V2_48K", "vits_config_array", "make_vits_weights",
    "make_vits_inputs", "make_vits_noise", "make_hubert_weights",
    "make_hubert_input", "coarse_pitch", "make_index", "make_queries",
    "make_rmvpe_weights", "make_rmvpe_input", "RMVPE_ENC", "RMVPE_INTER", "RMVPE_DEC", "make_speech_audio",
    "make_fcpe_weights",
]

# (sr, upsample_rates, upsample_kernels) of the two measured v2 generators.
# 40k uses the v1/40k decoder (configs/v1/40k.json); 48k is configs/v2/48k.json.
VITS_V2_40K = (40000, [10, 10, 2, 2], [16, 16, 4, 4])
VITS_V2_48K = (48000, [12, 10, 2, 2], [24, 20, 4, 4])

_HIDDEN = 192
_FILTER = 768
_PHONE = 768
_HEADS = 2
_LAYERS = 6
_WINDOW = 10
_GIN = 256
_UP0 = 512


def vits_config_array(sr: int = 40000) -> list:
    """Config array in the checkpoint layout of ``runtime/models/vits.py:174-177``."""
    sr_, rates, kernels = VITS_V2_48K if sr == 48000 else VITS_V2_40K
    return [1025, 32, _HIDDEN, _HIDDEN, _FILTER, _HEADS, _LAYERS, 3, 0, "1",
            [3, 7, 11], [[1, 3, 5], [1, 3, 5], [1, 3, 5]], list(rates), _UP0,
            list(kernels), 1, _GIN, sr_]


class _Gen:
    def __init__(self, seed: int):
        self.rs = np.random.RandomState(seed)

    def n(self, *shape, std=0.02):
        return (self.rs.standard_normal(shape) * std).astype(np.float32)

    def wn(self, d: dict, key: str, shape, gain: float):
        """weight_norm pair: v ~ N(0,0.02), g = gain * (1 + 0.1 N) per dim-0 row."""
        d[key + ".weight_v"] = self.n(*shape)
        g = gain * (1.0 + 0.1 * self.rs.standard_normal((shape[0], 1, 1)))
        d[key + ".weight_g"] = g.astype(np.float32)


def make_vits_weights(sr: int = 40000, seed: int = 0) -> dict:
    """Random-init ``SynthesizerTrnMs768NSFsid`` state dict (v2, 1 speaker).

    Key names and shapes follow the reference loader
    (``runtime/models/vits.py:166-249``, ``:499-538``, ``:962-1059``,
    ``:1086-1145``, ``:1285-1311``, ``:1390-1501``, ``:2133-2231``).
    """
    _, rates, kernels = VITS_V2_48K if sr == 48000 else VITS_V2_40K
    G = _Gen(seed)
    w: dict = {}
    h, f = _HIDDEN, _FILTER
    kc = h // _HEADS
    w["emb_g.weight"] = G.n(1, _GIN, std=0.5)
    w["enc_p.emb_phone.weight"] = G.n(h, _PHONE)
    w["enc_p.emb_phone.bias"] = G.n(h)
    w["enc_p.emb_pitch.weight"] = G.n(256, h)
    for i in range(_LAYERS):
        p = f"enc_p.encoder.attn_layers.{i}"
        for nm in ("conv_q", "conv_k", "conv_v", "conv_o"):
            w[f"{p}.{nm}.weight"] = G.n(h, h, 1, std=1.0 / math.sqrt(h))
            w[f"{p}.{nm}.bias"] = G.n(h)
        w[f"{p}.emb_rel_k"] = G.n(1, 2 * _WINDOW + 1, kc, std=kc ** -0.5)
        w[f"{p}.emb_rel_v"] = G.n(1, 2 * _WINDOW + 1, kc, std=kc ** -0.5)
        for nm in ("norm_layers_1", "norm_layers_2"):
            w[f"enc_p.encoder.{nm}.{i}.gamma"] = np.ones(h, np.float32)
            w[f"enc_p.encoder.{nm}.{i}.beta"] = np.zeros(h, np.float32)
        q = f"enc_p.encoder.ffn_layers.{i}"
        w[f"{q}.conv_1.weight"] = G.n(f, h, 3, std=1.0 / math.sqrt(3 * h))
        w[f"{q}.conv_1.bias"] = G.n(f)
        w[f"{q}.conv_2.weight"] = G.n(h, f, 3, std=1.0 / math.sqrt(3 * f))
        w[f"{q}.conv_2.bias"] = G.n(h)
    w["enc_p.proj.weight"] = G.n(2 * h, h, 1, std=0.5 / math.sqrt(h))
    w["enc_p.proj.bias"] = G.n(2 * h)
    half = h // 2
    for idx in (0, 2, 4, 6):
        p = f"flow.flows.{idx}"
        w[f"{p}.pre.weight"] = G.n(h, half, 1, std=1.0 / math.sqrt(half))
        w[f"{p}.pre.bias"] = G.n(h)
        G.wn(w, f"{p}.enc.cond_layer", (2 * h * 3, _GIN, 1), gain=1.0)
        w[f"{p}.enc.cond_layer.bias"] = G.n(2 * h * 3)
        for i in range(3):
            G.wn(w, f"{p}.enc.in_layers.{i}", (2 * h, h, 5), gain=1.0)
            w[f"{p}.enc.in_layers.{i}.bias"] = G.n(2 * h)
            out = 2 * h if i < 2 else h
            G.wn(w, f"{p}.enc.res_skip_layers.{i}", (out, h, 1), gain=0.5)
            w[f"{p}.enc.res_skip_layers.{i}.bias"] = G.n(out)
        w[f"{p}.post.weight"] = G.n(half, h, 1, std=0.3 / math.sqrt(h))
        w[f"{p}.post.bias"] = G.n(half)
    # ---- GeneratorNSF ----
    w["dec.conv_pre.weight"] = G.n(_UP0, h, 7, std=1.0 / math.sqrt(7 * h))
    w["dec.conv_pre.bias"] = G.n(_UP0)
    w["dec.cond.weight"] = G.n(_UP0, _GIN, 1, std=1.0 / math.sqrt(_GIN))
    w["dec.cond.bias"] = G.n(_UP0)
    w["dec.m_source.l_linear.weight"] = np.array([[0.9]], np.float32) + G.n(1, 1)
    w["dec.m_source.l_linear.bias"] = G.n(1)
    n_ups = len(rates)
    for i in range(n_ups):
        cin = _UP0 // (2 ** i)
        cout = cin // 2
        # convT weight [Cin, Cout, K]; norm is per input channel (dim 0).
        # Variance gain of a stride-r transposed conv ~ g^2 * Cin / (Cout * r).
        gain = math.sqrt(rates[i] * cout / cin) * 1.2
        G.wn(w, f"dec.ups.{i}", (cin, cout, kernels[i]), gain=gain)
        w[f"dec.ups.{i}.bias"] = G.n(cout)
        stride_f0 = int(np.prod(rates[i + 1:])) if i + 1 < n_ups else 1
        kn = stride_f0 * 2 if i + 1 < n_ups else 1
        w[f"dec.noise_convs.{i}.weight"] = G.n(cout, 1, kn, std=1.0 / math.sqrt(kn))
        w[f"dec.noise_convs.{i}.bias"] = G.n(cout)
        for j, k in enumerate((3, 7, 11)):
            base = f"dec.resblocks.{i * 3 + j}"
            for conv in ("convs1", "convs2"):
                for m in range(3):
                    G.wn(w, f"{base}.{conv}.{m}", (cout, cout, k), gain=0.8)
                    w[f"{base}.{conv}.{m}.bias"] = G.n(cout)
    w["dec.conv_post.weight"] = G.n(1, _UP0 // (2 ** n_ups), 7,
                                    std=0.6 / math.sqrt(7 * _UP0 // (2 ** n_ups)))
    return w


def coarse_pitch(f0: np.ndarray) -> np.ndarray:
    """Mel quantisation of f0 to the 1..255 coarse bins (``runtime/pipeline.py:424-483``)."""
    f0_min, f0_max = 50.0, 1100.0
    mel_min = 1127 * np.log(1 + f0_min / 700)
    mel_max = 1127 * np.log(1 + f0_max / 700)
    f0 = np.asarray(f0, dtype=np.float64)
    mel = 1127 * np.log(1 + f0 / 700)
    pos = mel > 0
    mel[pos] = (mel[pos] - mel_min) * 254 / (mel_max - mel_min) + 1
    mel = np.clip(mel, 1, 255)
    return np.rint(mel).astype(np.int64)


def make_vits_inputs(P: int, seed: int = 0, phone_dim: int = _PHONE):
    """One chunk of synthesizer inputs (BASELINE config 0 distribution).

    Returns ``phone [1,P,768] f32 ~N(0,1)``, ``pitch [1,P] int64`` (coarse bins of
    nsff0), ``nsff0 [1,P] f32 ~U(100,400) Hz`` with 10 % of frames zeroed
    (unvoiced), ``sid [1] int64 = 0``.
    """
    rs = np.random.RandomState(10_000 + seed)
    phone = rs.standard_normal((1, P, phone_dim)).astype(np.float32)
    f0 = rs.uniform(100.0, 400.0, size=P)
    f0[rs.uniform(size=P) < 0.1] = 0.0
    nsff0 = f0.astype(np.float32)[None, :]
    pitch = coarse_pitch(f0)[None, :]
    sid = np.zeros(1, np.int64)
    return phone, pitch, nsff0, sid


def make_vits_noise(P: int, upp: int, seed: int, hidden: int = _HIDDEN):
    """``nz [1,192,P]`` then ``ns [1,P*upp,1]`` from ``RandomState(seed)``.

    Same draw order as ``SynthesizerTrn._make_noise`` (``runtime/models/vits.py:2337-2350``).
    """
    rng = np.random.RandomState(seed)
    nz = rng.standard_normal((1, hidden, P)).astype(np.float32)
    ns = rng.standard_normal((1, P * upp, 1)).astype(np.float32)
    return nz, ns


def make_hubert_weights(seed: int = 0) -> dict:
    """Random-init HuBERT-base state dict with transformers key names.

    Keys follow the reference loader ``runtime/models/hubert.py:499-559``.
    """
    G = _Gen(20_000 + seed)
    sd: dict = {}
    ks = [10, 3, 3, 3, 3, 2, 2]
    cin = 1
    for i, k in enumerate(ks):
        sd[f"feature_extractor.conv_layers.{i}.conv.weight"] = G.n(
            512, cin, k, std=1.0 / math.sqrt(cin * k))
        cin = 512
    sd["feature_extractor.conv_layers.0.layer_norm.weight"] = np.ones(512, np.float32)
    sd["feature_extractor.conv_layers.0.layer_norm.bias"] = np.zeros(512, np.float32)
    sd["feature_projection.layer_norm.weight"] = np.ones(512, np.float32)
    sd["feature_projection.layer_norm.bias"] = np.zeros(512, np.float32)
    sd["feature_projection.projection.weight"] = G.n(768, 512)
    sd["feature_projection.projection.bias"] = G.n(768)
    sd["encoder.pos_conv_embed.conv.weight_g"] = (
        1.0 + 0.1 * G.rs.standard_normal((1, 1, 128))).astype(np.float32)
    sd["encoder.pos_conv_embed.conv.weight_v"] = G.n(768, 48, 128)
    sd["encoder.pos_conv_embed.conv.bias"] = G.n(768)
    sd["encoder.layer_norm.weight"] = np.ones(768, np.float32)
    sd["encoder.layer_norm.bias"] = np.zeros(768, np.float32)
    for i in range(12):
        p = f"encoder.layers.{i}."
        for nm in ("q_proj", "k_proj", "v_proj", "out_proj"):
            sd[p + f"attention.{nm}.weight"] = G.n(768, 768)
            sd[p + f"attention.{nm}.bias"] = G.n(768)
        sd[p + "layer_norm.weight"] = np.ones(768, np.float32)
        sd[p + "layer_norm.bias"] = np.zeros(768, np.float32)
        sd[p + "feed_forward.intermediate_dense.weight"] = G.n(3072, 768)
        sd[p + "feed_forward.intermediate_dense.bias"] = G.n(3072)
        sd[p + "feed_forward.output_dense.weight"] = G.n(768, 3072)
        sd[p + "feed_forward.output_dense.bias"] = G.n(768)
        sd[p + "final_layer_norm.weight"] = np.ones(768, np.float32)
        sd[p + "final_layer_norm.bias"] = np.zeros(768, np.float32)
    sd["final_proj.weight"] = G.n(256, 768)
    sd["final_proj.bias"] = G.n(256)
    return sd


def make_hubert_input(T: int = 160000, seed: int = 0) -> np.ndarray:
    """16 kHz waveform ``[1,T] f32 ~U(-0.5,0.5)``."""
    rs = np.random.RandomState(30_000 + seed)
    return rs.uniform(-0.5, 0.5, size=(1, T)).astype(np.float32)


def make_index(N: int, D: int = 768, seed: int = 0) -> np.ndarray:
    """Feature index ``[N,D] f32 ~N(0,1)`` (200000 x 768)."""
    rs = np.random.RandomState(40_000 + seed)
    return rs.standard_normal((N, D)).astype(np.float32)


def make_queries(F: int, D: int = 768, seed: int = 0) -> np.ndarray:
    """Retrieval queries ``[F,D] f32 ~N(0,1)`` (one per feature frame)."""
    rs = np.random.RandomState(50_000 + seed)
    return rs.standard_normal((F, D)).astype(np.float32)


# RMVPE E2E(4, 1, (2, 2)) channel plan (runtime/models/rmvpe.py:7-22):
# (in, out) per encoder / intermediate / decoder layer, 4 ConvBlockRes each.
RMVPE_ENC = [(1, 16), (16, 32), (32, 64), (64, 128), (128, 256)]
RMVPE_INTER = [(256, 512), (512, 512), (512, 512), (512, 512)]
RMVPE_DEC = [(512, 256), (256, 128), (128, 64), (64, 32), (32, 16)]


def make_rmvpe_weights(seed: int = 0) -> dict:
    """Random-init RMVPE state dict (He-scaled conv weights,
    BatchNorm statistics near (0, 1)).  Keys follow the reference's use of the
    checkpoint (``runtime/models/rmvpe.py:486-547``, ``:643-751``)."""
    G = _Gen(60_000 + seed)

    def conv(o, i, kh, kw):
        return G.n(o, i, kh, kw, std=math.sqrt(2.0 / (i * kh * kw)))

    def bn(sd, p, c):
        sd[p + ".weight"] = (1.0 + 0.1 * G.rs.standard_normal(c)).astype(np.float32)
        sd[p + ".bias"] = (0.1 * G.rs.standard_normal(c)).astype(np.float32)
        sd[p + ".running_mean"] = (0.1 * G.rs.standard_normal(c)).astype(np.float32)
        sd[p + ".running_var"] = G.rs.uniform(0.5, 1.5, c).astype(np.float32)
        sd[p + ".num_batches_tracked"] = np.zeros((), np.float32)

    def block(sd, p, cin, cout):
        sd[p + ".conv.0.weight"] = conv(cout, cin, 3, 3)
        bn(sd, p + ".conv.1", cout)
        sd[p + ".conv.3.weight"] = conv(cout, cout, 3, 3)
        bn(sd, p + ".conv.4", cout)
        if cin != cout:
            sd[p + ".shortcut.weight"] = conv(cout, cin, 1, 1)
            sd[p + ".shortcut.bias"] = (0.1 * G.rs.standard_normal(cout)).astype(np.float32)

    sd: dict = {}
    bn(sd, "unet.encoder.bn", 1)
    for i, (ci, co) in enumerate(RMVPE_ENC):
        for j in range(4):
            block(sd, f"unet.encoder.layers.{i}.conv.{j}", ci if j == 0 else co, co)
    for i, (ci, co) in enumerate(RMVPE_INTER):
        for j in range(4):
            block(sd, f"unet.intermediate.layers.{i}.conv.{j}", ci if j == 0 else co, co)
    for i, (ci, co) in enumerate(RMVPE_DEC):
        p = f"unet.decoder.layers.{i}"
        sd[p + ".conv1.0.weight"] = G.n(ci, co, 3, 3, std=math.sqrt(2.0 / (ci * 9 / 4)))
        bn(sd, p + ".conv1.1", co)
        for j in range(4):
            block(sd, f"{p}.conv2.{j}", 2 * co if j == 0 else co, co)
    sd["cnn.weight"] = conv(3, 16, 3, 3)
    sd["cnn.bias"] = (0.1 * G.rs.standard_normal(3)).astype(np.float32)
    Hh = 256
    a = 1.0 / math.sqrt(Hh)
    for suf in ("", "_reverse"):
        sd[f"fc.0.gru.weight_ih_l0{suf}"] = G.rs.uniform(-a, a, (3 * Hh, 384)).astype(np.float32)
        sd[f"fc.0.gru.weight_hh_l0{suf}"] = G.rs.uniform(-a, a, (3 * Hh, Hh)).astype(np.float32)
        sd[f"fc.0.gru.bias_ih_l0{suf}"] = G.rs.uniform(-a, a, 3 * Hh).astype(np.float32)
        sd[f"fc.0.gru.bias_hh_l0{suf}"] = G.rs.uniform(-a, a, 3 * Hh).astype(np.float32)
    sd["fc.1.weight"] = G.n(360, 512, std=1.0 / math.sqrt(512))
    sd["fc.1.bias"] = (-2.0 + 0.1 * G.rs.standard_normal(360)).astype(np.float32)
    return sd


def make_rmvpe_input(T: int = 160000, seed: int = 0) -> np.ndarray:
    """16 kHz mono ``[T] f32``: a harmonic tone on a random-walk f0 (80-300 Hz)
    plus white noise, 10 s by default."""
    rs = np.random.RandomState(70_000 + seed)
    f0 = np.clip(150.0 + np.cumsum(rs.standard_normal(T)) * 0.05, 80.0, 300.0)
    ph = 2 * np.pi * np.cumsum(f0) / 16000.0
    x = 0.3 * np.sin(ph) + 0.1 * np.sin(2 * ph) + 0.05 * np.sin(3 * ph) + 0.02 * rs.standard_normal(T)
    return x.astype(np.float32)


def make_speech_audio(seconds: float = 60.0, seed: int = 0, sr: int = 16000, silence_every: float = 8.0,
                      silence_len: float = 0.5, noise_db: float = -20.0) -> np.ndarray:
    """Speech-like 16 kHz audio ``[T] f32``: three
    harmonics (1, 1/2, 1/4) on an f0 random walk in 80-300 Hz (a step every
    10 ms, linear between steps), a slow amplitude envelope, pink noise at
    ``noise_db`` relative to the harmonic signal's RMS, and digital silences of
    ``silence_len`` s starting every ``silence_every`` s."""
    rs = np.random.RandomState(80_000 + seed)
    T = int(round(seconds * sr))
    nfr = T // 160 + 2
    walk = np.empty(nfr)
    f = rs.uniform(100.0, 250.0)
    for i in range(nfr):
        f = min(300.0, max(80.0, f + rs.standard_normal() * 4.0))
        walk[i] = f
    f0 = np.interp(np.arange(T) / 160.0, np.arange(nfr), walk)
    ph = 2.0 * np.pi * np.cumsum(f0) / sr
    env = 0.6 + 0.4 * np.sin(2.0 * np.pi * np.arange(T) / sr * 3.1 + rs.uniform(0, 2 * np.pi))
    x = env * (0.4 * np.sin(ph) + 0.2 * np.sin(2 * ph) + 0.1 * np.sin(3 * ph))
    spec = np.fft.rfft(rs.standard_normal(T))
    freqs = np.arange(spec.size, dtype=np.float64)
    freqs[0] = 1.0
    pink = np.fft.irfft(spec / np.sqrt(freqs), n=T)
    rms_x = np.sqrt(np.mean(x * x))
    pink *= rms_x * 10.0 ** (noise_db / 20.0) / max(np.sqrt(np.mean(pink * pink)), 1e-12)
    y = x + pink
    step, ln = int(silence_every * sr), int(silence_len * sr)
    for s in range(step, T, step):
        y[s:s + ln] = 0.0
    return y.astype(np.float32)


def make_fcpe_weights(seed: int = 0) -> dict:
    """Random-init FCPE (CFNaiveMelPE, conv-only) state dict with the keys the
    reference reads (``runtime/models/fcpe.py:237-302``): conv weights scaled by
    1/sqrt(fan_in), norm gains near 1, the output projection's weight-norm gain
    set to 2 so the 360 logits stay O(1) (an unsaturated sigmoid), and the
    cent table of the bundled model (360 bins from 32.7 Hz to 1975.5 Hz)."""
    rs = np.random.RandomState(95_000 + seed)

    def n(*shape, std):
        return (rs.standard_normal(shape) * std).astype(np.float32)

    sd = {
        "input_stack.0.weight": n(512, 128, 3, std=1.0 / math.sqrt(384)),
        "input_stack.0.bias": n(512, std=0.1),
        "input_stack.1.weight": (1.0 + n(512, std=0.1)).astype(np.float32),
        "input_stack.1.bias": n(512, std=0.1),
        "input_stack.3.weight": n(512, 512, 3, std=1.0 / math.sqrt(1536)),
        "input_stack.3.bias": n(512, std=0.1),
    }
    for i in range(6):
        p = f"net.encoder_layers.{i}.conformer.net"
        sd[p + ".0.weight"] = (1.0 + n(512, std=0.1)).astype(np.float32)
        sd[p + ".0.bias"] = n(512, std=0.1)
        sd[p + ".2.weight"] = n(2048, 512, 1, std=1.0 / math.sqrt(512))
        sd[p + ".2.bias"] = n(2048, std=0.1)
        sd[p + ".4.conv.weight"] = n(1024, 1, 31, std=1.0 / math.sqrt(31))
        sd[p + ".4.conv.bias"] = n(1024, std=0.1)
        sd[p + ".6.weight"] = n(512, 1024, 1, std=0.5 / math.sqrt(1024))
        sd[p + ".6.bias"] = n(512, std=0.1)
    sd["norm.weight"] = (1.0 + n(512, std=0.1)).astype(np.float32)
    sd["norm.bias"] = n(512, std=0.1)
    sd["output_proj.weight_v"] = n(360, 512, std=1.0)
    sd["output_proj.weight_g"] = np.full((360, 1), 2.0, np.float32)
    sd["output_proj.bias"] = (-1.0 + n(360, std=0.1)).astype(np.float32)
    sd["cent_table"] = np.linspace(1200.0 * np.log2(32.7 / 10.0), 1200.0 * np.log2(1975.5 / 10.0),
                                   360).astype(np.float32)
    return sd
