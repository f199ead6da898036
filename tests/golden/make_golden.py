"""Generate golden vectors by running the reference's own numpy CPU path.

Run in a container where the reference checkout is present::

    python tests/golden/make_golden.py [--ref /path/to/rvc-vulkan]

It imports ``runtime`` from the reference (read-only, ``RVC_BACKEND=numpy``),
replaces the checkpoint loaders with the seeded synthetic checkpoints of
``rvc_cuda.synthetic`` (the loaders read files; no checkpoints exist here),
runs ``SynthesizerTrn.infer_controlled`` / ``HubertEncoder.encode`` /
``RMVPE.infer_from_audio``, the
retrieval search (``runtime.retrieval.search_l2``) and the per-op numpy
kernels, and writes ``tests/golden/*.npz``.  Weights and inputs
are not stored: they are regenerated from the recorded seeds (legacy
``RandomState`` streams are frozen) and checked against recorded SHA-256
digests, so a drift in generation is detected rather than silently compared.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "rvc-vulkan_b200"))

from rvc_cuda import synthetic as syn  # noqa: E402


def digest(arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode())
        h.update(str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()


def weights_digest(w: dict) -> str:
    return digest([w[k] for k in sorted(w)])


# (name, sr, P frames, weight seed, input seed, noise seed)
VITS_CASES = [
    ("vits40k_p32", 40000, 32, 0, 1, 11),
    ("vits48k_p24", 48000, 24, 1, 2, 12),
    ("vits40k_p7", 40000, 7, 0, 3, 13),     # P < window+1: sliced rel-embeddings
]
# (name, T samples, weight seed, input seed)
HUBERT_CASES = [
    ("hubert_t8000", 8000, 0, 1),
    ("hubert_t3201", 3201, 0, 2),           # odd length: ragged conv strides
]
# partial synthesis (infer with skip_head / return_length):
# (name, sr, P, weight seed, input seed, noise seed, head, length)
PARTIAL_CASES = [
    ("vits40k_p96_part", 40000, 96, 0, 4, 14, 50, 20),   # interior segment, flow from frame 10
    ("vits48k_p40_part", 48000, 40, 1, 5, 15, 5, 30),    # head < pads: segment starts at 0
]
# (name, T samples, weight seed, input seed)
RMVPE_CASES = [
    ("rmvpe_t16000", 16000, 0, 1),          # 101 frames -> U-Net on 128
    ("rmvpe_t6401", 6401, 0, 2),            # 41 frames: padded to 64, odd length
]
# (name, F queries, N index rows, D, k, index seed, query seed)
RETRIEVAL_CASES = [
    ("ret_f200_n20000", 200, 20000, 768, 8, 0, 0),   # several 4096-row merge chunks
    ("ret_f64_n3000_d256", 64, 3000, 256, 8, 1, 1),  # v1 feature width
    ("ret_f37_n5", 37, 5, 768, 8, 2, 2),             # N < k: k' = N
    ("ret_f9_n1000_d60", 9, 1000, 60, 3, 3, 3),      # D not a multiple of 16, k = 3
]


def run_vits(runtime_vits, name, sr, P, wseed, iseed, nseed, meta):
    w = syn.make_vits_weights(sr, wseed)
    cfg = syn.vits_config_array(sr)
    runtime_vits._load_ckpt = lambda path: {"weight": w, "config": cfg}
    net = runtime_vits.SynthesizerTrn("synthetic.pth")
    phone, pitch, nsff0, sid = syn.make_vits_inputs(P, iseed)
    nz, ns = syn.make_vits_noise(P, net.cfg.upp, nseed)
    rec = {}
    enc_cls = runtime_vits._TextEncoder
    flow_cls = runtime_vits._FlowBlock
    orig_stats, orig_rev = enc_cls.stats, flow_cls.reverse

    def stats(self, x):
        rec["enc_h"] = np.array(x[0])
        m, logs = orig_stats(self, x)
        rec["enc_m"], rec["enc_logs"] = np.array(m[0].T), np.array(logs[0].T)
        return m, logs

    def reverse(self, z, x_mask, g):
        out = orig_rev(self, z, x_mask, g)
        rec["flow_z"] = np.array(out[0].T)
        return out

    enc_cls.stats, flow_cls.reverse = stats, reverse
    try:
        wav = net.infer_controlled(phone, pitch, nsff0, sid, nz, ns)
    finally:
        enc_cls.stats, flow_cls.reverse = orig_stats, orig_rev
    rec["wave"] = np.asarray(wav, np.float32).reshape(-1)
    np.savez_compressed(os.path.join(HERE, name + ".npz"), **rec)
    meta[name] = {
        "kind": "vits", "sr": sr, "P": P, "weight_seed": wseed, "input_seed": iseed,
        "noise_seed": nseed, "upp": int(net.cfg.upp),
        "weights_sha256": weights_digest(w),
        "inputs_sha256": digest([phone, pitch, nsff0, sid, nz, ns]),
    }


def run_hubert(runtime_hubert, name, T, wseed, iseed, meta):
    sd = syn.make_hubert_weights(wseed)
    x = syn.make_hubert_input(T, iseed)
    with tempfile.TemporaryDirectory() as d:
        open(os.path.join(d, "pytorch_model.bin"), "wb").close()
        runtime_hubert.load_pth = lambda path: sd
        enc = runtime_hubert.HubertEncoder(d)
        feats = enc._feature_extractor(x)
        out = enc.encode(x, version=2)
        out1 = enc.encode(x, version=1)
    np.savez_compressed(os.path.join(HERE, name + ".npz"),
                        conv=np.asarray(feats[0], np.float32),
                        out=np.asarray(out[0], np.float32),
                        out_v1=np.asarray(out1[0], np.float32))
    meta[name] = {"kind": "hubert", "T": T, "weight_seed": wseed, "input_seed": iseed,
                  "weights_sha256": weights_digest(sd), "inputs_sha256": digest([x])}


def run_partial(runtime_vits, name, sr, P, wseed, iseed, nseed, head, length, meta):
    """``SynthesizerTrn._infer_partial`` (the skip_head path of ``infer``) on seeded inputs."""
    w = syn.make_vits_weights(sr, wseed)
    cfg = syn.vits_config_array(sr)
    phone, pitch, nsff0, sid = syn.make_vits_inputs(P, iseed)
    upp = int(np.prod(cfg[12]))
    nz, ns = syn.make_vits_noise(P, upp, nseed)
    runtime_vits._load_ckpt = lambda path: {"weight": w, "config": cfg}
    m = runtime_vits.SynthesizerTrn("synthetic.pth")
    wav = m._infer_partial(phone, pitch, nsff0, sid, nz, ns, head, length)
    np.savez_compressed(os.path.join(HERE, name + ".npz"), wave=np.asarray(wav, np.float32).reshape(-1))
    meta[name] = {"kind": "vits_partial", "sr": sr, "P": P, "upp": upp, "weight_seed": wseed, "input_seed": iseed,
                  "noise_seed": nseed, "head": head, "length": length, "weights_sha256": weights_digest(w),
                  "inputs_sha256": digest([phone, pitch, nsff0, sid, nz, ns])}


def run_rmvpe(runtime_rmvpe, name, T, wseed, iseed, meta):
    """``RMVPE.infer_from_audio`` pieces: log-mel, salience (``mel2hidden``), f0."""
    sd = syn.make_rmvpe_weights(wseed)
    x = syn.make_rmvpe_input(T, iseed)
    with tempfile.TemporaryDirectory() as d:
        runtime_rmvpe.load_pth = lambda path: sd
        m = runtime_rmvpe.RMVPE(os.path.join(d, "rmvpe.pt"))
    mel = m._extract_mel(x)
    hidden = m.mel2hidden(mel)
    f0 = m.infer_from_audio(x)
    np.savez_compressed(os.path.join(HERE, name + ".npz"), mel=mel[0], salience=hidden[0],
                        argmax=np.argmax(hidden[0], axis=1).astype(np.int64), f0=f0)
    meta[name] = {"kind": "rmvpe", "T": T, "weight_seed": wseed, "input_seed": iseed,
                  "weights_sha256": weights_digest(sd), "inputs_sha256": digest([x])}


def run_retrieval(retrieval, name, F, N, D, k, iseed, qseed, meta):
    """The reference's ``search_l2`` and ``weighted_blend`` (``runtime/retrieval.py:35-108``)
    plus the pipeline blend written exactly as ``runtime/pipeline.py:547-551`` does it."""
    db = syn.make_index(N, D, iseed)
    q = syn.make_queries(F, D, qseed)
    sc, ix = retrieval.search_l2(q, db, k=k)
    blk = db[ix]
    w = np.square(1.0 / sc)
    w /= np.maximum(w.sum(axis=1, keepdims=True), 1e-12)
    pipe = np.sum(blk * w[:, :, None], axis=1)
    wb = retrieval.weighted_blend(q, db, k=k)
    # blends of the first 16 queries keep the fixture small; all scores/indices are stored
    np.savez_compressed(os.path.join(HERE, name + ".npz"), scores=sc, inds=ix, blend=pipe[:16],
                        weighted=wb[:16])
    meta[name] = {"kind": "retrieval", "F": F, "N": N, "D": D, "k": k, "index_seed": iseed, "query_seed": qseed,
                  "inputs_sha256": digest([db, q])}


# (name, N, D, nlist, F, seed, far-centroid edge case)
IVF_CASES = [
    ("ivf_n8000_d256", 8000, 256, 32, 120, 1, False),
    ("ivf_n40_d16_edge", 40, 16, 8, 30, 2, True),
]


def run_ivf(name, N, D, nlist, F, seed, edge, meta):
    """The reference's IVF search (``runtime/pipeline.py:_ivf_strict_search``)
    over an ``IVFIndex`` trained by its own mini-batch k-means, for nprobe 1
    and 3, and the pipeline's IVF blend through ``Pipeline._vc_prepare`` with
    the ``IVFIndex`` as the index (index_rate 0.75).  Centroids and bucket
    assignments are stored (the k-means is the reference's code)."""
    from runtime import pipeline as rp  # noqa: PLC0415
    from runtime.ivf_index import IVFIndex  # noqa: PLC0415
    sys.path.insert(0, HERE)
    import pipeline_fakes as pf  # noqa: PLC0415
    vecs = syn.make_index(N, D, 100 + seed)
    q = syn.make_queries(F, D, 200 + seed)
    ivf = IVFIndex(dim=D, nlist=nlist, nprobe=1)
    ivf.train(vecs, seed=seed)
    if edge:  # two centroids far from every row: empty buckets; queries next to one of them
        c = ivf.centroids.copy()
        c[-1] = 0.0
        c[-1, 0] = 40.0
        c[-2] = 0.0
        c[-2, 1] = -40.0
        ivf.set_centroids(c)
        q[:5] = c[-1] + 0.01 * q[:5]
    ivf.add(vecs)
    rec = {"centroids": ivf.centroids, "assignments": ivf._assignments.astype(np.int32)}
    for npb in (1, 3):
        sc, ix = rp._ivf_strict_search(ivf, q, k=8, nprobe=npb)
        rec[f"scores_p{npb}"], rec[f"inds_p{npb}"] = sc, ix
    feats = (q[None] * 0.5).astype(np.float32)
    P = F
    pitch = np.ones((1, 2 * P), np.int64) * 60
    pitchf = np.full((1, 2 * P), 150.0, np.float32)
    pitchf[0, ::3] = 0.0
    pipe = rp.Pipeline(40000, pf.config())
    prep = pipe._vc_prepare(None, 0, np.zeros(2 * P * 160 + 400, np.float32), pitch, pitchf, [0.0, 0.0, 0.0], ivf,
                            None, 0.75, 2, 0.33, feats=feats)
    rec["prep_feats"] = prep["feats"]
    # the two-path retrieval mix (brute_mix, runtime/pipeline.py:521-566)
    for tag, mode, bm in (("bm_ivf", "ivf", 0.3), ("bm_brute", "brute", 0.4)):
        prep = pipe._vc_prepare(None, 0, np.zeros(2 * P * 160 + 400, np.float32), pitch, pitchf, [0.0, 0.0, 0.0],
                                ivf, None, 0.75, 2, 0.33, feats=feats, retrieval_mode=mode, brute_mix=bm)
        rec[f"prep_{tag}"] = prep["feats"][:, ::7]  # every 7th frame keeps the fixture small
    np.savez_compressed(os.path.join(HERE, name + ".npz"), **rec)
    meta[name] = {"kind": "ivf", "N": N, "D": D, "nlist": int(ivf.nlist), "F": F, "seed": seed, "edge": edge,
                  "inputs_sha256": digest([vecs, q])}


# (name, T samples, weight seed, input seed)
FCPE_CASES = [
    ("fcpe_t24000", 24000, 0, 3),
    ("fcpe_t3001", 3001, 0, 4),
    ("fcpe_t400", 400, 0, 5),                 # shorter than the right pad: constant padding
]


def run_fcpe(name, T, wseed, iseed, meta):
    """The reference's numpy ``FCPE`` (``runtime/models/fcpe.py:165-369``) with the
    seeded synthetic checkpoint: log-mel, sigmoid latent, argmax and f0."""
    from runtime.models import fcpe as rf  # noqa: PLC0415
    sd = syn.make_fcpe_weights(wseed)
    x = syn.make_rmvpe_input(T, iseed)
    rf.load_pth = lambda path: {"model": sd}
    with tempfile.TemporaryDirectory() as d:
        open(os.path.join(d, "fcpe.pt"), "wb").close()
        m = rf.FCPE(os.path.join(d, "fcpe.pt"))
    mel = m._wav2mel(x)
    lat = m._latent(mel)
    f0 = m.infer(x)
    f0_argmax = m.infer(x, decoder_mode="argmax")
    # Pipeline.get_f0(..., "fcpe") with this model (runtime/pipeline.py:451-483)
    from runtime import pipeline as rp  # noqa: PLC0415
    sys.path.insert(0, HERE)
    import pipeline_fakes as pf  # noqa: PLC0415
    pipe = rp.Pipeline(40000, pf.config())
    pipe.model_fcpe = m
    coarse, f0bak = pipe.get_f0(x.astype(np.float64), T // 160 + 1, 3, "fcpe")
    np.savez_compressed(os.path.join(HERE, name + ".npz"), mel=mel[0], latent=lat[0],
                        argmax=lat[0].argmax(axis=1).astype(np.int64), f0=f0, f0_argmax=f0_argmax,
                        pipe_coarse=coarse, pipe_f0bak=f0bak)
    meta[name] = {"kind": "fcpe", "T": T, "weight_seed": wseed, "input_seed": iseed,
                  "weights_sha256": weights_digest(sd), "inputs_sha256": digest([x])}


def run_ops(nn, meta):
    """Per-op vectors from ``runtime.nn``'s numpy kernels (``_conv1d_numpy`` etc.)."""
    rs = np.random.RandomState(4242)
    rec = {}
    cases = []
    conv_cases = [  # (B, C, T, O, K, stride, pad, dil)
        (1, 5, 37, 7, 3, 1, 1, 1), (2, 16, 64, 8, 7, 1, (3, 3), 2),
        (1, 3, 50, 4, 10, 5, 0, 1), (1, 8, 33, 8, 11, 1, (25, 25), 5),
        (1, 4, 9, 6, 5, 2, (2, 1), 1), (1, 2, 3, 3, 5, 1, 0, 1),
    ]
    for i, (B, C, T, O, K, s, p, d) in enumerate(conv_cases):
        x = rs.standard_normal((B, C, T)).astype(np.float32)
        w = rs.standard_normal((O, C, K)).astype(np.float32)
        b = rs.standard_normal(O).astype(np.float32)
        rec[f"conv1d_{i}_x"], rec[f"conv1d_{i}_w"], rec[f"conv1d_{i}_b"] = x, w, b
        rec[f"conv1d_{i}_y"] = nn._conv1d_numpy(x, w, b, s, p, d)
        cases.append({"op": "conv1d", "i": i, "stride": s,
                      "padding": list(p) if isinstance(p, tuple) else p, "dilation": d})
    convt_cases = [(1, 6, 11, 4, 16, 10, 3), (2, 8, 7, 5, 4, 2, 1), (1, 3, 5, 2, 24, 12, 6)]
    for i, (B, Ci, T, Co, K, s, p) in enumerate(convt_cases):
        x = rs.standard_normal((B, Ci, T)).astype(np.float32)
        w = rs.standard_normal((Ci, Co, K)).astype(np.float32)
        b = rs.standard_normal(Co).astype(np.float32)
        rec[f"convt_{i}_x"], rec[f"convt_{i}_w"], rec[f"convt_{i}_b"] = x, w, b
        rec[f"convt_{i}_y"] = nn._conv_transpose1d_numpy(x, w, b, s, p, 0, 1)
        cases.append({"op": "conv_transpose1d", "i": i, "stride": s, "padding": p})
    x = (rs.standard_normal((3, 17, 192)) * 3 + 1).astype(np.float32)
    g = rs.standard_normal(192).astype(np.float32)
    bt = rs.standard_normal(192).astype(np.float32)
    rec["ln_x"], rec["ln_g"], rec["ln_b"] = x, g, bt
    from runtime import backend  # numpy backend: the reference formula
    rec["ln_y"] = backend.layer_norm(x, g, bt, 1e-5)
    sx = (rs.standard_normal((4, 33)) * 10).astype(np.float32)
    sx[0, :] += 1000.0
    rec["sm_x"], rec["sm_y"] = sx, backend.softmax(sx)
    gx = (rs.standard_normal(4096) * 3).astype(np.float32)
    rec["gelu_x"] = gx
    from runtime.models import hubert as rh
    rec["gelu_y"] = rh.gelu_erf(gx)
    rec["leaky_x"] = gx
    rec["leaky_y"] = nn.leaky_relu(gx, 0.1)
    np.savez_compressed(os.path.join(HERE, "ops.npz"), **rec)
    meta["ops"] = {"kind": "ops", "cases": cases}


def run_dsp(meta):
    """Pipeline signal processing through the reference's own call sites:
    ``signal.filtfilt(_BH, _AH, .)`` (``runtime/pipeline.py:49``, ``:765``),
    ``change_rms`` (``:164``), ``Pipeline._vc_prepare`` with given features
    (x2 interpolation, frame alignment, protect; ``:488-614``) and whole
    ``Pipeline.pipeline`` runs (``:697``) with the deterministic model
    stand-ins of ``pipeline_fakes`` (split points recovered from the offsets of
    the segments handed to ``get_f0``; int16 output)."""
    from runtime import pipeline as rp  # noqa: PLC0415
    sys.path.insert(0, HERE)
    import pipeline_fakes as pf  # noqa: PLC0415
    rec, cases = {}, {}
    audio = syn.make_speech_audio(0.5, seed=1)
    rec["hp_speech"] = rp.signal.filtfilt(rp._BH, rp._AH, audio)
    edge = np.random.RandomState(91_001).standard_normal(19).astype(np.float32)
    rec["hp_edge_x"], rec["hp_edge"] = edge, rp.signal.filtfilt(rp._BH, rp._AH, edge)
    x64 = np.random.RandomState(91_002).standard_normal(300) * 0.3
    rec["hp_f64_x"], rec["hp_f64"] = x64, rp.signal.filtfilt(rp._BH, rp._AH, x64)
    cases["hp_speech"] = {"seconds": 0.5, "seed": 1, "inputs_sha256": digest([audio])}

    d1 = syn.make_speech_audio(0.6, seed=2)
    d2 = (0.8 * np.sin(np.arange(24000) * 0.03) * np.random.RandomState(91_003).uniform(0.2, 1.0, 24000)
          ).astype(np.float32)
    rec["rms_d2"], rec["rms_out"] = d2, rp.change_rms(d1, d2, 16000, 40000, 0.25)
    rec["rms_small_d2"] = d2[:700].copy()
    rec["rms_small_out"] = rp.change_rms(d1, rec["rms_small_d2"], 16000, 48000, 0.6)
    cases["rms"] = {"seconds": 0.6, "seed": 2, "inputs_sha256": digest([d1])}

    rs = np.random.RandomState(91_004)
    feats = rs.standard_normal((1, 30, 256)).astype(np.float32)
    pitch = rs.randint(1, 256, size=(1, 57)).astype(np.int64)
    pitchf = rs.uniform(100, 300, size=(1, 57)).astype(np.float32)
    pitchf[0, rs.rand(57) < 0.3] = 0.0
    pipe = rp.Pipeline(40000, pf.config())
    prep = pipe._vc_prepare(None, 0, np.zeros(60 * 160 + 400, np.float32), pitch, pitchf, [0.0, 0.0, 0.0], None,
                            None, 0, 1, 0.33, feats=feats)
    rec.update(prep_feats=feats, prep_pitch=pitch, prep_pitchf=pitchf, prep_out=prep["feats"],
               prep_out_pitch=prep["pitch"], prep_out_pitchf=prep["pitchf"])

    for name, kw in PIPE_CASES:
        a = syn.make_speech_audio(kw["seconds"], seed=kw["seed"], silence_every=kw["silence_every"])
        pipe = rp.Pipeline(40000, pf.config(x_query=kw["x_query"]))
        pipe.model_rmvpe = pf.FakeRmvpe()
        starts = []
        orig = pipe.get_f0

        def get_f0(x, *args, _orig=orig, _starts=starts):
            _starts.append(x.__array_interface__["data"][0])
            return _orig(x, *args)

        pipe.get_f0 = get_f0
        sr, out = pipe.pipeline(pf.FakeHubert(D=768), pf.FakeSynth(gain=kw["gain"]), 0, a, [0.0, 0.0, 0.0],
                                kw["f0_up_key"], kw.get("f0", "rmvpe"), None, 0, True, 40000,
                                kw.get("resample_sr", 0), kw["rms"], 2, kw["protect"], slice_length=kw["slice_length"])
        assert sr == 40000
        item = np.dtype(np.float64).itemsize
        rec[name + "_split"] = np.array([(p - starts[0]) // item - pipe.t_pad for p in starts[1:]], np.int64)
        if out.size > 200_000:  # long case: every 101st sample keeps the fixture small
            rec[name + "_int16_every101"] = out[::101].copy()
        else:
            rec[name + "_int16"] = out
        cases[name] = dict(kw, inputs_sha256=digest([a]), out_len=int(out.size))
    # pm f0 (runtime/dsp/f0.py:24) and Pipeline.get_f0(..., "pm") with its padding and post-processing
    from runtime.dsp.f0 import f0_autocorrelation  # noqa: PLC0415
    a = syn.make_speech_audio(1.5, seed=6, silence_every=0.6, silence_len=0.2)
    a[3000:3400] += (0.3 * np.random.RandomState(91_005).standard_normal(400)).astype(np.float32)
    rec["pm_f0"] = f0_autocorrelation(a.astype(np.float64), 16000, voicing_threshold=0.6, f0_min=50, f0_max=1100,
                                      time_step=0.01)
    pipe = rp.Pipeline(40000, pf.config())
    p_len = a.size // 160 + 3
    rec["pm_coarse"], rec["pm_f0bak"] = pipe.get_f0(a.astype(np.float64), p_len, 4, "pm")
    cases["pm"] = {"seconds": 1.5, "seed": 6, "p_len": p_len, "inputs_sha256": digest([a])}
    # output resampling (runtime/dsp/resample.py:129), the three methods
    from runtime.dsp.resample import resample  # noqa: PLC0415
    wv = (0.6 * np.sin(np.arange(12001) * 0.05) + 0.2 * np.random.RandomState(91_006).standard_normal(12001)
          ).astype(np.float32)
    rec["rs_x"] = wv
    for meth in ("fft", "linear", "sinc"):
        rec[f"rs_{meth}_48k"] = resample(wv, 40000, 48000, method=meth)
        rec[f"rs_{meth}_16k"] = resample(wv, 40000, 16000, method=meth)
    np.savez_compressed(os.path.join(HERE, "dsp.npz"), **rec)
    meta["dsp"] = {"kind": "dsp", "cases": cases, "scipy": __import__("scipy").__version__}


# whole-pipeline cases with the stand-in models (40 kHz output)
PIPE_CASES = [
    ("pipe_split", {"seconds": 8.0, "seed": 3, "silence_every": 2.1, "x_query": 1, "slice_length": 2.0,
                    "rms": 0.25, "protect": 0.33, "gain": 1.3, "f0_up_key": 2}),
    ("pipe_voiced", {"seconds": 3.0, "seed": 5, "silence_every": 100.0, "x_query": 1, "slice_length": 1.0,
                     "rms": 0.5, "protect": 0.2, "gain": 0.7, "f0_up_key": 0}),
    ("pipe_whole", {"seconds": 1.2, "seed": 4, "silence_every": 8.0, "x_query": 6, "slice_length": 0,
                    "rms": 1.0, "protect": 0.5, "gain": 1.3, "f0_up_key": -3}),
    ("pipe_resample_pm", {"seconds": 1.3, "seed": 10, "silence_every": 8.0, "x_query": 6, "slice_length": 0,
                          "rms": 0.5, "protect": 0.33, "gain": 1.3, "f0_up_key": 1, "f0": "pm",
                          "resample_sr": 48000}),
    ("pipe_60s", {"seconds": 60.0, "seed": 0, "silence_every": 8.0, "x_query": 6, "slice_length": 0,
                  "rms": 0.25, "protect": 0.33, "gain": 1.3, "f0_up_key": 0}),
]


def run_refruns(ref, meta):
    """The reference's own ``SynthesizerTrn``, ``Pipeline.pipeline`` and
    ``VC.vc_single`` on seeded weights (``reference_runs.py --backend numpy``,
    in a child process: the operator backend is chosen once per process)."""
    import subprocess  # noqa: PLC0415

    out = os.path.join(HERE, "refruns.npz")
    env = dict(os.environ, RVC_REFERENCE=ref)
    subprocess.run([sys.executable, os.path.join(HERE, "reference_runs.py"), "--backend", "numpy", "--out", out],
                   check=True, env=env)
    sys.path.insert(0, HERE)
    import reference_runs as rr  # noqa: PLC0415

    runs = np.load(out)
    for case in ("pipeline", "vc"):
        gap, coarse = runs[case + "_margins"]
        if not (gap >= rr.MIN_RET_GAP and coarse >= rr.MIN_COARSE_MARGIN):
            raise SystemExit(f"refruns: the {case} case has a decision margin below the bar "
                             f"(retrieval gap {gap}, coarse {coarse}); change its inputs")
    meta["refruns"] = {"kind": "reference_runs", "seed": rr.SEED, "clip_s": rr.CLIP_S, "clip_seed": rr.CLIP_SEED,
                       "index_n": rr.INDEX_N, "index_seed": rr.INDEX_SEED, "pipeline": rr.PIPE_KW}


def run_config4(ref, meta):
    """The reference's ``Pipeline.pipeline`` on config 4's 60 s clip with its
    own numpy models (``reference_runs.py --cases config4``, ~10 minutes)."""
    import subprocess  # noqa: PLC0415

    out = os.path.join(HERE, "config4.npz")
    env = dict(os.environ, RVC_REFERENCE=ref)
    subprocess.run([sys.executable, os.path.join(HERE, "reference_runs.py"), "--backend", "numpy", "--out", out,
                    "--cases", "config4"], check=True, env=env)
    sys.path.insert(0, HERE)
    import reference_runs as rr  # noqa: PLC0415

    gap, coarse = np.load(out)["config4_margins"]
    if not (gap >= rr.MIN_RET_GAP and coarse >= rr.MIN_COARSE_MARGIN):
        raise SystemExit(f"config4: a decision margin is below the bar (retrieval gap {gap}, coarse {coarse})")
    meta["config4"] = {"kind": "reference_runs", "seconds": rr.C4_SECONDS, "seed": rr.C4_SEED,
                       "stride": rr.C4_STRIDE, "index_n": rr.INDEX_N, "index_seed": rr.INDEX_SEED,
                       "fixed_seed": rr.SEED, "pipeline": rr.config4_kwargs()}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("RVC_REFERENCE", ""),
                    help="checkout of the reference (default: $RVC_REFERENCE, else the oracle/_ref copy)")
    ap.add_argument("--only", choices=["vits", "hubert", "ops", "retrieval", "rmvpe", "partial", "dsp", "ivf", "fcpe",
                                       "refruns", "config4"], default=None,
                    help="regenerate one family and keep the other fixtures")
    args = ap.parse_args()
    if not args.ref:
        sys.path.insert(0, ROOT)
        from oracle import reference as oref  # noqa: PLC0415

        args.ref = oref.root() or ""
    if not args.ref:
        ap.error("no reference: pass --ref <checkout> or set RVC_REFERENCE (or run make -C oracle ref)")
    os.environ["RVC_BACKEND"] = "numpy"
    sys.path.insert(0, args.ref)
    from runtime import nn  # noqa: PLC0415
    from runtime.models import hubert as runtime_hubert  # noqa: PLC0415
    from runtime.models import vits as runtime_vits  # noqa: PLC0415
    import numba  # noqa: PLC0415
    import threadpoolctl  # noqa: PLC0415

    meta = {"numpy": np.__version__, "numba": numba.__version__,
            "blas": [i.get("internal_api") for i in threadpoolctl.threadpool_info()]}
    if args.only is not None:
        with open(os.path.join(HERE, "golden.json")) as f:
            meta = json.load(f)
    if args.only in (None, "vits"):
        for c in VITS_CASES:
            run_vits(runtime_vits, *c, meta)
    if args.only in (None, "hubert"):
        for c in HUBERT_CASES:
            run_hubert(runtime_hubert, *c, meta)
    if args.only in (None, "ops"):
        run_ops(nn, meta)
    if args.only in (None, "partial"):
        for c in PARTIAL_CASES:
            run_partial(runtime_vits, *c, meta)
    if args.only in (None, "rmvpe"):
        from runtime.models import rmvpe as runtime_rmvpe  # noqa: PLC0415
        for c in RMVPE_CASES:
            run_rmvpe(runtime_rmvpe, *c, meta)
    if args.only in (None, "dsp"):
        run_dsp(meta)
    if args.only in (None, "fcpe"):
        for c in FCPE_CASES:
            run_fcpe(*c, meta)
    if args.only in (None, "ivf"):
        for c in IVF_CASES:
            run_ivf(*c, meta)
    if args.only in (None, "retrieval"):
        from runtime import retrieval  # noqa: PLC0415
        for c in RETRIEVAL_CASES:
            run_retrieval(retrieval, *c, meta)
    if args.only in (None, "refruns"):
        run_refruns(args.ref, meta)
    if args.only in (None, "config4"):
        run_config4(args.ref, meta)
    with open(os.path.join(HERE, "golden.json"), "w") as f:
        json.dump(meta, f, indent=1, sort_keys=True)
    print("wrote", sorted(k for k in meta if k not in ("numpy", "numba", "blas")))


if __name__ == "__main__":
    main()
