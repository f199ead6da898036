"""The offline conversion pipeline with its signal processing on the device.

``Pipeline`` mirrors the reference's ``runtime.pipeline.Pipeline``
(``runtime/pipeline.py:368``): the same constructor ``(tgt_sr, config)``, the
same ``get_f0`` and ``pipeline(...)`` signatures and return value
``(tgt_sr, int16 audio)``, the same chunking.  The models are the duck-typed
objects the reference's pipeline takes (``runtime/pipeline.py:15-25``):
``model.encode`` / ``encode_batch`` (``CudaHubert``), ``net_g.infer`` /
``prep_dec`` + ``decode_batch`` (``CudaSynthesizer``) and
``self.model_rmvpe.infer_from_audio`` (``CudaRmvpe``) or
``self.model_fcpe.infer`` (``CudaFcpe``).  The steps between the
models run on the device through ``rvc_cuda.dsp``: the 48 Hz high-pass, the
silence split, the retrieval blend (``CudaIndex``), the x2 interpolation and
the protect blend, ``change_rms`` and the int16 conversion.

Host-side glue that stays in numpy: the reflect padding and slicing of the
chunks, the frame alignment of pitch arrays (``:572-603``) and the f0
post-processing of ``get_f0`` (``:468-482``, a few thousand values per call).

``brute_mix != 0`` (a blend of the IVF and brute-force retrievals) runs on the
host-buffer path: both blends come from the device index and are mixed in
float32 in the reference's order.
"""

from __future__ import annotations

import os
import time
from typing import Optional

import numpy as np

from . import dsp

__all__ = ["Pipeline"]

_WINDOW = 160
_K_SEARCH = 8


def _as_version(version):
    """1 / 2 from 1, 2, "v1", "v2" (``runtime/pipeline.py:1281-1288``)."""
    if version in ("v1", "v2"):
        return 1 if version == "v1" else 2
    v = int(version)
    if v not in (1, 2):
        raise ValueError(f"version must be 1 or 2, got {version!r}")
    return v


def _align(arr, n):
    """Repeat the last frame or cut to ``n`` frames (``runtime/pipeline.py:582-603``)."""
    m = arr.shape[1]
    if m == n:
        return arr
    if m < n:
        return np.concatenate([arr, np.repeat(arr[:, -1:], n - m, axis=1)], axis=1)
    return arr[:, :n]


class Pipeline:
    """Device pipeline with the reference ``Pipeline``'s interface."""

    def __init__(self, tgt_sr, config):
        self.x_pad, self.x_query, self.x_center, self.x_max = (config.x_pad, config.x_query, config.x_center,
                                                               config.x_max)
        self.is_half = False
        self.sr = 16000
        self.window = _WINDOW
        self.t_pad = self.sr * self.x_pad
        self.t_pad_tgt = tgt_sr * self.x_pad
        self.t_pad2 = self.t_pad * 2
        self.t_query = self.sr * self.x_query
        self.t_center = self.sr * self.x_center
        self.t_max = self.sr * self.x_max
        self.device = getattr(config, "device", None)

    # ------------------------------------------------------------------ f0
    def get_f0(self, x, p_len, f0_up_key, f0_method):
        """f0 of a segment (``rmvpe`` through ``self.model_rmvpe``, ``fcpe``
        through ``self.model_fcpe``, ``pm`` through the device
        autocorrelation) and the reference's
        post-processing (``runtime/pipeline.py:408-483``): unvoiced frames
        linearly interpolated, transposed by ``f0_up_key`` semitones, then the
        mel quantisation to 1..255.  Returns ``(f0_coarse int32, f0 float32)``."""
        if f0_method not in ("pm", "rmvpe", "fcpe"):
            raise ValueError(f"Unsupported F0 method: {f0_method}")
        return self._f0_post(self._f0_raw(x, p_len, f0_method), f0_up_key)

    def _f0_raw(self, x, p_len, f0_method):
        """The f0 estimator's Hz curve of a segment (``runtime/pipeline.py:428-462``)."""
        f0_min, f0_max = 50, 1100
        if f0_method == "pm":                                          # :428-441
            f0 = np.asarray(dsp.f0_autocorrelation(np.asarray(x, dtype=np.float64), self.sr, voicing_threshold=0.6,
                                                   f0_min=f0_min, f0_max=f0_max, time_step=0.01), dtype=np.float64)
            pad_size = (p_len - len(f0) + 1) // 2
            right = p_len - len(f0) - pad_size
            if pad_size > 0 or right > 0:
                f0 = np.pad(f0, (pad_size, right), mode="constant")
        elif f0_method == "fcpe":                                      # :451-462
            if not hasattr(self, "model_fcpe"):
                raise RuntimeError("Pipeline.model_fcpe must be set (a CudaFcpe, or any object with "
                                   "infer(x, sr, decoder_mode, threshold))")
            f0 = np.asarray(self.model_fcpe.infer(np.asarray(x, dtype=np.float32), sr=16000,
                                                  decoder_mode="local_argmax", threshold=0.006), dtype=np.float64)
        else:
            if not hasattr(self, "model_rmvpe"):
                raise RuntimeError("Pipeline.model_rmvpe must be set (a CudaRmvpe, or any object with "
                                   "infer_from_audio(x, thred))")
            f0 = np.asarray(self.model_rmvpe.infer_from_audio(np.asarray(x, dtype=np.float32), thred=0.03),
                            dtype=np.float64)
        return f0

    @staticmethod
    def _f0_post(f0, f0_up_key):
        """Unvoiced frames interpolated, transposition, mel quantisation to
        1..255 (``runtime/pipeline.py:468-482``)."""
        f0_min, f0_max = 50, 1100
        f0_mel_min = 1127 * np.log(1 + f0_min / 700)
        f0_mel_max = 1127 * np.log(1 + f0_max / 700)
        f0 = np.array(f0, dtype=np.float64)
        uv = f0 == 0
        if uv.any():
            voiced = np.where(~uv)[0]
            if voiced.size:
                f0[uv] = np.interp(np.where(uv)[0], voiced, f0[voiced])
        f0 *= pow(2, f0_up_key / 12)
        f0bak = f0.astype(np.float32).copy()
        f0_mel = 1127 * np.log(1 + f0 / 700)
        f0_mel[f0_mel > 0] = (f0_mel[f0_mel > 0] - f0_mel_min) * 254 / (f0_mel_max - f0_mel_min) + 1
        f0_mel = np.clip(f0_mel, 1, 255)
        return np.rint(f0_mel).astype(np.int32), f0bak

    # ------------------------------------------------------------------ index
    @staticmethod
    def _resolve_index(file_index, index_rate):
        """The device index for ``file_index`` (``runtime/pipeline.py:1227-1256``):
        a ``CudaIndex``, an ``[N, D]`` array, an object with ``ntotal`` /
        ``reconstruct_n`` (the reference's ``FeatureIndex``: brute force) or an
        ``IVFIndex`` (``vectors_by_rows``: inverted-file search), or None."""
        from . import retrieval  # noqa: PLC0415
        if index_rate == 0 or file_index is None or (isinstance(file_index, str) and file_index == ""):
            return None
        if isinstance(file_index, retrieval.CudaIndex):
            return file_index if file_index.N > 0 else None
        if isinstance(file_index, str):
            raise NotImplementedError("index files are loaded by the caller: pass the index object or a CudaIndex")
        if getattr(file_index, "vectors_by_rows", None) is not None:
            if getattr(file_index, "ntotal", 0) <= 0:
                return None
            if str(getattr(file_index, "metric", "L2")).upper() == "IP":
                raise NotImplementedError("inner-product (IP) indexes are not supported by the L2 blend")
            return retrieval._ivf_for(file_index)
        if isinstance(file_index, np.ndarray):
            vecs = file_index
        elif hasattr(file_index, "reconstruct_n") and hasattr(file_index, "ntotal"):
            if file_index.ntotal <= 0:
                return None
            vecs = file_index.reconstruct_n(0, file_index.ntotal)
        else:
            return None
        return retrieval._index_for(vecs)

    # ------------------------------------------------------------------ chunk
    def _vc_prepare(self, sid, audio_len, pitch, pitchf, feats, index, index_rate, protect, times,
                    retrieval_mode="ivf", brute_mix=0.0):
        """Per-chunk preparation (``runtime/pipeline.py:488-614``) on the device:
        retrieval blend, x2 interpolation of ``feats`` (and of the unblended
        ``feats0`` when protecting), frame alignment, protect blend."""
        t0 = time.perf_counter()
        feats = np.asarray(feats, dtype=np.float32)
        protecting = protect < 0.5 and pitch is not None and pitchf is not None
        feats0 = feats if protecting else None
        if index is not None and index_rate != 0 and brute_mix != 0:  # :521-566, the two-path blend
            feats = self._mixed_blend(index, feats, index_rate, retrieval_mode, float(brute_mix))
        elif index is not None and index_rate != 0:                 # :517-566
            if index.nlist and retrieval_mode != "brute":             # IVF index: strict bucket search
                feats = index.ivf_blend(feats[0], k=_K_SEARCH, feats=feats[0], index_rate=index_rate)[None]
            else:                                                     # brute force over every row
                feats = index.blend(feats[0], k=_K_SEARCH, mode="pipeline", feats=feats[0],
                                    index_rate=index_rate)[None]
        feats = dsp.interpolate_linear(feats, scale_factor=2, axis=1)
        if protecting:
            feats0 = dsp.interpolate_linear(feats0, scale_factor=2, axis=1)
        t1 = time.perf_counter()
        if pitch is not None and pitchf is not None:
            n = feats.shape[1]
            pitch = _align(pitch, n)
            pitchf = _align(pitchf, n)
        if protecting:
            pitchf = _align(pitchf, feats.shape[1])
            feats = dsp.protect_blend(feats, feats0, pitchf, protect)
        times[0] += t1 - t0
        return {"feats": feats, "pitch": pitch, "pitchf": pitchf, "sid_arr": np.asarray([sid], dtype=np.int64)}

    @staticmethod
    def _mixed_blend(index, feats, index_rate, retrieval_mode, brute_mix):
        """``brute_mix != 0`` (``runtime/pipeline.py:521-566``): the IVF blend (the
        strict bucket search; the brute-force blend again when the index has no
        IVF structure) and the brute-force blend over every row, both on the
        device; mixed as ``(1 - m) * main + m * other`` (main = IVF, or the
        brute force under ``retrieval_mode="brute"``), then
        ``blend * index_rate + feats * (1 - index_rate)``, in float32 as there."""
        q = feats[0]
        brute = index.blend(q, k=_K_SEARCH, mode="pipeline")
        ivf = index.ivf_blend(q, k=_K_SEARCH) if index.nlist else brute
        m = float(brute_mix)  # Python scalars against float32 arrays, as there
        if retrieval_mode == "brute":
            blend = (1.0 - m) * brute + m * ivf
        else:
            blend = (1.0 - m) * ivf + m * brute
        return (blend[None, :, :] * float(index_rate) + feats * (1 - float(index_rate))).astype(np.float32)

    # ------------------------------------------------------------------ whole
    def pipeline(self, model, net_g, sid, audio, times, f0_up_key, f0_method, file_index, index_rate, if_f0,
                 tgt_sr, resample_sr, rms_mix_rate, version, protect, progress_cb=None, slice_length=0,
                 retrieval_mode="ivf", brute_mix=0.0):
        """Offline conversion of 16 kHz ``audio`` (``runtime/pipeline.py:697-1213``).
        Returns ``(tgt_sr, int16 audio)``."""
        if not if_f0:
            raise NotImplementedError("only f0-guided models are supported (as in the reference)")
        index = self._resolve_index(file_index, index_rate)
        version = _as_version(version)
        t_max = self.t_max
        try:
            slice_length = float(slice_length or 0)
        except (TypeError, ValueError):
            slice_length = 0
        if slice_length > 0:
            t_max = int(slice_length * self.sr)

        audio = np.asarray(audio, dtype=np.float32)
        audio = dsp.highpass(audio)                                   # float64, :765

        opt_ts = []
        if audio.shape[0] + 2 * (self.window // 2) > t_max:           # :769-790
            step = min(self.t_center, t_max)
            opt_ts = dsp.split_points(audio, self.t_query, step, self.window)

        audio_pad = np.pad(audio, (self.t_pad, self.t_pad), mode="reflect")   # :799 / :819
        total = len(opt_ts) + 1
        bounds, s = [], 0
        for t in opt_ts:                                              # :840-846
            t = t // self.window * self.window
            bounds.append((s, t))
            s = t
        bounds.append((s, None))
        blocks = []                                                   # (idx, s0, e0, chunk audio)
        for idx, (s0, e0) in enumerate(bounds):
            blk = audio_pad[s0:] if e0 is None else audio_pad[s0:e0 + self.t_pad2 + self.window]
            if blk.shape[0] >= self.window * 10:
                blocks.append((idx, s0, e0, np.asarray(blk, dtype=np.float32)))
        noise = self._prefetch_noise(model, net_g, [b[3].shape[0] for b in blocks])

        # the two-path retrieval mix (brute_mix) runs on the host-buffer path
        ctx = None if (brute_mix and index is not None and index_rate != 0) else self._device_chain(model, net_g, index)
        f0_model = getattr(self, "model_fcpe" if f0_method == "fcpe" else "model_rmvpe", None)
        f0_ctx = getattr(f0_model, "ctx", None)
        if ctx is not None and f0_method != "pm" and f0_ctx is not None and f0_ctx is not ctx:
            # the f0 model has its own stream: extract f0 on a host thread while the
            # device chain runs HuBERT, retrieval and interpolation
            from concurrent.futures import ThreadPoolExecutor  # noqa: PLC0415
            ex = ThreadPoolExecutor(max_workers=1, thread_name_prefix="rvc-f0")
            fut = ex.submit(self._f0_all, audio_pad, opt_ts, f0_up_key, f0_method, times)
            ex.shutdown(wait=False)
            if progress_cb is not None:
                progress_cb(0, total, "split into %d chunks" % total)
            return tgt_sr, self._convert_on_device(ctx, model, net_g, index, audio, blocks,
                                                   lambda: self._chunk_pitches(blocks, *fut.result()), noise, sid,
                                                   version, index_rate, protect, tgt_sr, resample_sr, rms_mix_rate,
                                                   times, retrieval_mode, brute_mix, progress_cb, total)
        pitch, pitchf = self._f0_all(audio_pad, opt_ts, f0_up_key, f0_method, times)
        if progress_cb is not None:
            progress_cb(0, total, "split into %d chunks" % total)
        pitches = self._chunk_pitches(blocks, pitch, pitchf)

        if ctx is not None:
            return tgt_sr, self._convert_on_device(ctx, model, net_g, index, audio, blocks, lambda: pitches, noise, sid,
                                                   version,
                                                   index_rate, protect, tgt_sr, resample_sr, rms_mix_rate, times,
                                                   retrieval_mode, brute_mix, progress_cb, total)
        feats_all = self._encode(model, [b[3] for b in blocks], version)
        preps = [self._vc_prepare(sid, b[3].shape[0], p[0], p[1], f, index, index_rate, protect, times,
                                  retrieval_mode, brute_mix) for b, p, f in zip(blocks, pitches, feats_all)]
        t2 = time.perf_counter()
        waves = self._decode(net_g, preps, noise)
        times[2] += time.perf_counter() - t2

        results = [None] * len(bounds)
        for done, ((idx, *_), w) in enumerate(zip(blocks, waves), 1):
            w = np.asarray(w, dtype=np.float32).reshape(-1)
            results[idx] = w[self.t_pad_tgt:-self.t_pad_tgt]
            if progress_cb is not None:
                progress_cb(done, total, "chunk %d/%d" % (done, total))
        audio_opt = np.concatenate([r for r in results if r is not None])
        if rms_mix_rate != 1:
            audio_opt = dsp.change_rms(audio, audio_opt, 16000, tgt_sr, rms_mix_rate)
        if tgt_sr != resample_sr >= 16000:                             # :1204-1205
            audio_opt = dsp.resample(audio_opt, tgt_sr, resample_sr, method="fft")
        return tgt_sr, dsp.to_int16(audio_opt)

    def _f0_all(self, audio_pad, opt_ts, f0_up_key, f0_method, times):
        """f0 of every split segment, concatenated (``runtime/pipeline.py:795-816``)."""
        t1 = time.perf_counter()
        seg_pts = [0] + [o + self.t_pad for o in opt_ts] + [audio_pad.shape[0]]
        segs, cores = [], []
        for si in range(len(seg_pts) - 1):
            ap, bp = seg_pts[si], seg_pts[si + 1]
            b = min(bp + self.t_pad2 + self.window, audio_pad.shape[0])
            segs.append(audio_pad[ap:b])
            cores.append(max(1, (bp - ap) // self.window))
        model = getattr(self, "model_rmvpe", None)
        if f0_method == "rmvpe" and len(segs) > 1 and hasattr(model, "infer_many"):
            # the segments are independent calls: run them concurrently
            raws = model.infer_many([np.asarray(g, dtype=np.float32) for g in segs], thred=0.03)
            outs = [self._f0_post(r, f0_up_key) for r in raws]
        else:
            outs = [self.get_f0(g, g.shape[0] // self.window, f0_up_key, f0_method) for g in segs]
        pitch_parts, pitchf_parts = [], []
        for (pi, pfi), core_n in zip(outs, cores):
            pitch_parts.append(pi[:core_n])
            pitchf_parts.append(pfi[:core_n])
        pitch = np.concatenate(pitch_parts)[None, :]
        pitchf = np.concatenate(pitchf_parts).astype(np.float32)[None, :]
        times[1] += time.perf_counter() - t1
        return pitch, pitchf

    def _chunk_pitches(self, blocks, pitch, pitchf):
        """Each chunk's slice of the frame-level pitch (``runtime/pipeline.py:903-916``)."""
        out = []
        for idx, s0, e0, _ in blocks:
            if e0 is None:
                out.append((pitch[:, s0 // self.window:], pitchf[:, s0 // self.window:]))
            else:
                out.append((pitch[:, s0 // self.window:(e0 + self.t_pad2) // self.window],
                            pitchf[:, s0 // self.window:(e0 + self.t_pad2) // self.window]))
        return out

    # ------------------------------------------------------------------ device-resident path
    @staticmethod
    def _device_chain(model, net_g, index):
        """The context every stage shares when the models are this library's
        (``CudaHubert``, ``CudaSynthesizer``, ``CudaIndex`` on one device), else None."""
        from .hubert import CudaHubert  # noqa: PLC0415
        from .synth import CudaSynthesizer  # noqa: PLC0415
        if not (isinstance(model, CudaHubert) and isinstance(net_g, CudaSynthesizer)) or model.ctx is not net_g.ctx:
            return None
        if index is not None and getattr(index, "ctx", None) is not model.ctx:
            return None
        return model.ctx

    def _convert_on_device(self, ctx, model, net_g, index, audio, blocks, pitches_fn, noise, sid, version,
                           index_rate, protect, tgt_sr, resample_sr, rms_mix_rate, times, retrieval_mode, brute_mix,
                           progress_cb, total):
        """The chunk loop with the features and waveforms resident in HBM.  Phase
        A (no f0 needed): per chunk the audio goes up, HuBERT, the retrieval blend
        and the x2 interpolations run on device buffers.  Then the chunks' pitch
        (``pitches_fn``, which may wait for f0 extracted concurrently on another
        stream); phase B: protect blend, synthesizer, the trimmed waveform into
        one output buffer.  Finally change_rms and the int16 conversion on the
        device, one copy down.  The same kernels as the host-buffer path, so the
        same result."""
        if index is not None and index_rate != 0 and brute_mix != 0:
            raise NotImplementedError("brute_mix != 0 is not on the device path")
        D = 256 if version == 1 else 768
        upp, H = net_g.upp, net_g.hidden
        bufs = []

        def alloc(nbytes):
            p = ctx.alloc(max(16, int(nbytes)))
            bufs.append(p)
            return p

        def al(n):
            return (int(n) + 255) // 256 * 256

        try:
            plan, n_out, need = [], 0, 0
            for (idx, s0, e0, blk) in blocks:
                L = int(model.out_frames(blk.shape[0]))
                P = 2 * L
                keep = max(0, P * upp - 2 * self.t_pad_tgt)
                plan.append([blk, L, P, keep, 0, 0])
                n_out += keep
                need += al(4 * blk.shape[0]) + al(4 * P) + al(8 * P) + al(8)
            mix = rms_mix_rate != 1 and n_out > 0
            if mix:
                need += al(4 * np.asarray(audio).size)
            # uploads go through a page-locked staging buffer and are enqueued
            # without waiting for the stream (the final download waits for all)
            stage_buf, stage_off = self._pinned("stage", need), [0]

            def up(dptr, arr, dtype):
                a = np.ascontiguousarray(arr, dtype=dtype).reshape(-1)
                v = stage_buf.view(dtype, a.size, stage_off[0])
                v[...] = a
                stage_off[0] += al(a.nbytes)
                ctx.h2d_async(dptr, v)

            d_out = alloc(4 * n_out)
            d_a = 0
            if mix:                                                        # change_rms input, up early
                n_a = np.asarray(audio).size
                d_a = alloc(4 * n_a)
                up(d_a, audio, np.float32)
            for item in plan:                                              # phase A
                blk, L, P = item[0], item[1], item[2]
                t0 = time.perf_counter()
                T = blk.shape[0]
                d_x = alloc(4 * T)
                up(d_x, blk, np.float32)
                d_f = alloc(4 * L * D)
                model.encode_device(d_x, 1, T, version, d_f)
                d_m = d_f
                if index is not None and index_rate != 0:                 # :517-566
                    d_m = alloc(4 * L * D)
                    index.blend_device(d_f, L, d_f, index_rate, d_m, k=_K_SEARCH,
                                       ivf=bool(index.nlist) and retrieval_mode != "brute")
                d_ph = alloc(4 * P * D)
                dsp.interpolate_device(ctx, d_m, L, D, 2, d_ph, P)
                d_f0 = 0
                if protect < 0.5:
                    d_f0 = alloc(4 * P * D)
                    dsp.interpolate_device(ctx, d_f, L, D, 2, d_f0, P)
                item[4], item[5] = d_ph, d_f0
                times[0] += time.perf_counter() - t0
            pitches = pitches_fn()
            off = 0
            for done, (item, (p, pf)) in enumerate(zip(plan, pitches), 1):  # phase B
                blk, L, P, keep, d_ph, d_f0 = item
                t1 = time.perf_counter()
                pitch, pitchf = _align(p, P), _align(pf, P)                # :582-603
                d_pf = alloc(4 * P)
                up(d_pf, pitchf[0], np.float32)
                if protect < 0.5:                                          # :594-608
                    dsp.protect_device(ctx, d_ph, d_f0, d_pf, P, D, protect, d_ph)
                if noise is not None and noise[done - 1][0] == P:
                    nz, ns = noise[done - 1][1].result()
                else:
                    nz, ns = net_g.make_noise(P)
                d_p, d_sid = alloc(8 * P), alloc(8)
                d_nz, d_ns, d_w = alloc(4 * H * P), alloc(4 * P * upp), alloc(4 * P * upp)
                up(d_p, pitch[0], np.int64)
                up(d_sid, [sid], np.int64)
                for d, z in ((d_nz, nz), (d_ns, ns)):
                    z = np.asarray(z)
                    if z.dtype == np.float32 and z.flags.c_contiguous:
                        ctx.h2d_async(d, z)  # page-locked noise from the prefetch, or staged by the driver
                    else:
                        ctx.h2d(d, np.ascontiguousarray(z, dtype=np.float32))
                net_g.infer_device(1, P, d_ph, d_p, d_pf, d_sid, d_nz, d_ns, d_w)
                if keep:                                                   # [t_pad_tgt : -t_pad_tgt]
                    ctx.d2d(d_out + 4 * off, d_w + 4 * self.t_pad_tgt, 4 * keep)
                off += keep
                times[2] += time.perf_counter() - t1
                if progress_cb is not None:
                    progress_cb(done, total, "chunk %d/%d" % (done, total))
            if mix:
                dsp.change_rms_device(ctx, d_a, n_a, 16000, d_out, n_out, tgt_sr, rms_mix_rate, d_out)
            if tgt_sr != resample_sr >= 16000:
                host = np.empty(n_out, np.float32)
                if n_out:
                    ctx.d2h(host, d_out)
                return dsp.to_int16(dsp.resample(host, tgt_sr, resample_sr, method="fft"))
            out = np.empty(n_out, np.int16)
            if n_out:
                d_i = alloc(2 * n_out)
                dsp.to_int16_device(ctx, d_out, n_out, d_i)
                ctx.d2h(out, d_i)
            return out
        finally:
            for b in bufs:
                ctx.free(b)

    # ------------------------------------------------------------------ models
    @staticmethod
    def _encode(model, audios, version):
        """HuBERT features of every chunk: one ``encode_batch`` call when the
        model offers it (chunk results equal per-chunk ``encode``), else
        ``encode`` per chunk."""
        if not audios:
            return []
        if hasattr(model, "encode_batch") and len(audios) > 1:
            return [np.asarray(f, dtype=np.float32).reshape(1, -1, np.shape(f)[-1])
                    for f in model.encode_batch([a[None, :] for a in audios], version=version)]
        return [np.asarray(model.encode(a[None, :], version=version), dtype=np.float32) for a in audios]

    def _pinned(self, name, nbytes):
        """A page-locked host buffer of at least ``nbytes``, kept for reuse
        across calls (a call's asynchronous uploads from it end with the
        call's final device-to-host copy)."""
        from ._lib import PinnedBuffer  # noqa: PLC0415
        cache = self.__dict__.setdefault("_pin", {})
        buf = cache.get(name)
        if buf is None or buf.nbytes < nbytes:
            if buf is not None:
                buf.close()
            buf = cache[name] = PinnedBuffer(int(nbytes * 1.25) + 4096)
        return buf

    def _prefetch_noise(self, model, net_g, chunk_lengths):
        """Draw every chunk's synthesizer noise on host threads while the
        device runs f0 and HuBERT (``RandomState`` fills release the GIL),
        into page-locked buffers when the synthesizer is this library's, so
        the uploads overlap device work.  Needs the frame count before
        encoding: ``model.out_frames(T)`` (``CudaHubert``) and
        ``net_g.make_noise`` (``CudaSynthesizer``)."""
        if not (hasattr(net_g, "make_noise") and hasattr(net_g, "prep_dec") and hasattr(net_g, "decode_batch")
                and hasattr(model, "out_frames")) or not chunk_lengths:
            return None
        from concurrent.futures import ThreadPoolExecutor  # noqa: PLC0415

        from .synth import CudaSynthesizer  # noqa: PLC0415
        pin = isinstance(net_g, CudaSynthesizer)
        # each chunk draws from its own RandomState(seed), so the chunks are
        # independent: one thread per chunk (up to the host's cores)
        workers = max(1, min(len(chunk_lengths), os.cpu_count() or 1, 8))
        ex = ThreadPoolExecutor(max_workers=workers, thread_name_prefix="rvc-noise")
        jobs = []
        for i, n in enumerate(chunk_lengths):
            P = 2 * int(model.out_frames(n))
            if pin:
                nh, nn = net_g.hidden * P, P * net_g.upp
                buf = self._pinned(f"noise{i}", 4 * (nh + nn))
                out = (buf.view(np.float32, nh, 0), buf.view(np.float32, nn, 4 * nh))
                jobs.append((P, ex.submit(net_g.make_noise, P, None, out)))
            else:
                jobs.append((P, ex.submit(net_g.make_noise, P)))
        ex.shutdown(wait=False)
        return jobs

    @staticmethod
    def _decode(net_g, preps, noise=None):
        """Waveforms of every chunk: ``prep_dec`` + one ``decode_batch`` when the
        synthesizer offers them (with the prefetched noise where its frame count
        matches), else ``infer`` per chunk."""
        if hasattr(net_g, "prep_dec") and hasattr(net_g, "decode_batch") and (len(preps) > 1 or noise):
            dps = []
            for i, p in enumerate(preps):
                kw = {}
                if noise is not None and noise[i][0] == p["feats"].shape[1]:
                    kw["noise"] = noise[i][1].result()
                dps.append(net_g.prep_dec(p["feats"], p["pitch"], p["pitchf"], p["sid_arr"], **kw))
            return net_g.decode_batch(dps)
        return [np.asarray(net_g.infer(np.asarray(p["feats"], dtype=np.float32), p["pitch"], p["pitchf"],
                                       p["sid_arr"], phone_gpu=None))[0, 0] for p in preps]
