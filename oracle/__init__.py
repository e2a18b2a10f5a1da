"""TEST INFRASTRUCTURE ONLY -- ctypes front end of the two CPU checkers.

* ``port``: ``oracle/libs2oracle.so``, our plain-C restatement of the
  reference hot path (``oracle/s2_oracle.c``; always built by ``build()``).
* ``ref``: ``oracle/_ref/libs2ref.so``, the reference's own CPU layer code
  (``src/layers/seedvr2_dit_block.cpp``, ``dynamic_framewise_spatial_attention.cpp``)
  compiled unmodified against an ncnn-API shim (``oracle/ref_harness.cpp``).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's cpu_baseline /
``--impl reference`` legs may use this package, and only as the checker or the
timed CPU baseline. The product library never imports it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PORT_SO = os.path.join(HERE, "libs2oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libs2ref.so")
HEAD_DIM = 128

_f32p = ctypes.POINTER(ctypes.c_float)
_i32p = ctypes.POINTER(ctypes.c_int)
_u8p = ctypes.POINTER(ctypes.c_ubyte)


def reference_root() -> str | None:
    """Root of the reference source tree: $S2_REFERENCE_ROOT, else the
    ``reference_path`` recorded in the repository's BASELINE.json; None when
    neither names an existing tree (e.g. on a GPU box, which uses the
    prebuilt oracle/_ref)."""
    root = os.environ.get("S2_REFERENCE_ROOT")
    if not root:
        try:
            import json
            with open(os.path.join(os.path.dirname(HERE), "BASELINE.json")) as f:
                root = json.load(f).get("reference_path")
        except (OSError, ValueError):
            root = None
    return root if root and os.path.isdir(os.path.join(root, "src")) else None


def build(ref_root: str | None = None) -> None:
    """Compile the restatement, and the reference build when its tree exists."""
    ref_root = ref_root or reference_root()
    subprocess.run(["make", "-s", "-C", HERE, "port"], check=True)
    if ref_root:
        subprocess.run(["make", "-s", "-C", HERE, "ref", f"REF={ref_root}"], check=True)


def _ptr(a, t=_f32p):
    if a is None:
        return None
    return a.ctypes.data_as(t)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


class _Lib:
    def __init__(self, path: str):
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        self.path = path
        self.lib = ctypes.CDLL(path)


class Port(_Lib):
    """The C restatement (``oracle/s2_oracle.c``)."""

    def __init__(self, path: str = PORT_SO):
        super().__init__(path)
        L = self.lib
        L.s2o_make_windows.restype = ctypes.c_int
        L.s2o_make_windows.argtypes = [ctypes.c_int] * 7 + [_i32p, ctypes.c_int]
        L.s2o_round_bf16.restype = ctypes.c_float
        L.s2o_round_bf16.argtypes = [ctypes.c_float]
        L.s2o_window_attention.restype = ctypes.c_int
        L.s2o_window_attention.argtypes = (
            [_f32p, ctypes.c_int, _f32p, ctypes.c_int]
            + [ctypes.c_int] * 8 + [ctypes.c_float]
            + [_f32p] * 5 + [ctypes.c_int, ctypes.c_int, ctypes.c_int, _u8p, ctypes.c_int]
            + [_f32p] * 6)
        L.s2o_vae_attention.restype = ctypes.c_int
        L.s2o_vae_attention.argtypes = [ctypes.c_int] * 4 + [_f32p] * 11 + [ctypes.c_int] * 3 + [_f32p]
        L.s2o_vae_attention_tokens.restype = ctypes.c_int
        L.s2o_vae_attention_tokens.argtypes = ([ctypes.c_int] * 4 + [_f32p] * 11 + [ctypes.c_int]
                                               + [ctypes.POINTER(ctypes.c_int)] + [ctypes.c_int] * 2 + [_f32p])

    def group_norm(self, x, bias, weight, threads=0):
        """DynamicFramewiseGroupNorm on x [C, T, H, W]."""
        x = _f32(x)
        C, T, H, W = x.shape
        y = np.zeros_like(x)
        L = self.lib
        L.s2o_group_norm.restype = ctypes.c_int
        L.s2o_group_norm.argtypes = [ctypes.c_int] * 4 + [_f32p] * 3 + [ctypes.c_int, _f32p]
        rc = L.s2o_group_norm(C, T, H, W, _ptr(_f32(bias)), _ptr(_f32(weight)), _ptr(x),
                              int(threads or os.cpu_count() or 1), _ptr(y))
        if rc != 0:
            raise ValueError(f"s2o_group_norm failed: {rc}")
        return y

    def space_time_shuffle(self, x, bias, weight, threads=0):
        """DynamicSpaceTimeShuffle: x [Cin, T, H, W], weight [P, Cin] -> [Cin, T', 2H, 2W]."""
        x = _f32(x)
        C, T, H, W = x.shape
        P = int(np.asarray(bias).size)
        tr = P // C // 4
        y = np.zeros((C, T * tr - 1 if tr > 1 else T, 2 * H, 2 * W), np.float32)
        L = self.lib
        L.s2o_space_time_shuffle.restype = ctypes.c_int
        L.s2o_space_time_shuffle.argtypes = [ctypes.c_int] * 5 + [_f32p] * 3 + [ctypes.c_int, _f32p]
        rc = L.s2o_space_time_shuffle(C, P, T, H, W, _ptr(_f32(bias)), _ptr(_f32(weight)), _ptr(x),
                                      int(threads or os.cpu_count() or 1), _ptr(y))
        if rc != 0:
            raise ValueError(f"s2o_space_time_shuffle failed: {rc}")
        return y

    def conv3d(self, x, weight, bias=None, stride=(1, 1, 1), dilation=(1, 1, 1), pad=(0, 0, 0, 0, 0, 0),
               pad_value=0.0, threads=0):
        """Convolution3D: x [Cin, T, H, W], weight [Cout, Cin, kd, kh, kw];
        pad = (front, top, left, behind, bottom, right)."""
        x = _f32(x)
        weight = _f32(weight)
        C, T, H, W = x.shape
        Co, Ci, kd, kh, kw = weight.shape
        assert Ci == C
        L = self.lib
        L.s2o_conv3d.restype = ctypes.c_int
        L.s2o_conv3d.argtypes = ([ctypes.c_int] * 20 + [ctypes.c_float] + [_f32p] * 3 + [ctypes.c_int, _f32p]
                                 + [_i32p] * 3)
        od, oh, ow = ctypes.c_int(0), ctypes.c_int(0), ctypes.c_int(0)
        args = [C, T, H, W, Co, kd, kh, kw, *stride, *dilation, *pad, ctypes.c_float(pad_value),
                _ptr(None if bias is None else _f32(bias)), _ptr(weight), _ptr(x), int(threads or os.cpu_count() or 1)]
        if L.s2o_conv3d(*args, None, ctypes.byref(od), ctypes.byref(oh), ctypes.byref(ow)) != 0:
            raise ValueError("s2o_conv3d: bad arguments")
        y = np.zeros((Co, od.value, oh.value, ow.value), np.float32)
        L.s2o_conv3d(*args, _ptr(y), ctypes.byref(od), ctypes.byref(oh), ctypes.byref(ow))
        return y

    def make_windows(self, T, H, W, shifted, override=(0, 0, 0)):
        n = self.lib.s2o_make_windows(T, H, W, int(shifted), *override, None, 0)
        out = np.zeros((max(n, 1), 6), dtype=np.int32)
        self.lib.s2o_make_windows(T, H, W, int(shifted), *override, _ptr(out, _i32p), n)
        return out[:n]

    def window_attention(self, vid_qkv, txt_qkv, shape, heads, gammas, freqs, shifted,
                         override=(0, 0, 0), eps=1e-5, round_out=True, heads_range=None,
                         window_mask=None, threads=0, packed=False):
        """Returns (vid_out [L,dim], txt_out [Lt,dim], packed dict or None)."""
        T, H, W = shape
        vid_qkv, txt_qkv = _f32(vid_qkv), _f32(txt_qkv)
        L, Lt = vid_qkv.shape[0], txt_qkv.shape[0]
        dim = heads * HEAD_DIM
        g = [_f32(x) for x in gammas]
        fr = _f32(freqs)
        vo = np.zeros((L, dim), np.float32)
        to = np.zeros((Lt, dim), np.float32)
        pk = None
        if packed:
            wins = self.make_windows(T, H, W, shifted, override)
            rows = int(sum((w[1] - w[0]) * (w[3] - w[2]) * (w[5] - w[4]) + Lt for w in wins))
            pk = {k: np.zeros((rows, dim), np.float32) for k in "qkvo"}
        hb, he = heads_range if heads_range else (0, heads)
        mask = None if window_mask is None else np.ascontiguousarray(window_mask, dtype=np.uint8)
        rc = self.lib.s2o_window_attention(
            _ptr(vid_qkv), L, _ptr(txt_qkv), Lt, T, H, W, heads, int(shifted), *override,
            ctypes.c_float(eps), *[_ptr(x) for x in g], _ptr(fr), int(round_out), hb, he,
            _ptr(mask, _u8p), int(threads or os.cpu_count() or 1), _ptr(vo), _ptr(to),
            *([_ptr(pk[k]) for k in "qkvo"] if pk else [None] * 4))
        if rc != 0:
            raise ValueError(f"s2o_window_attention failed: {rc}")
        return vo, to, pk

    def vae_attention(self, x, weights, frames=None, threads=0):
        """x [C,T,H,W]; weights dict with the reference's load_model keys."""
        x = _f32(x)
        C, T, H, W = x.shape
        fb, fe = frames if frames else (0, T)
        y = np.zeros_like(x)
        order = ["norm_bias", "norm_weight", "k_bias", "k_weight", "out_bias", "out_weight",
                 "q_bias", "q_weight", "v_bias", "v_weight"]
        ws = [_f32(weights[k]) for k in order]
        rc = self.lib.s2o_vae_attention(C, T, H, W, *[_ptr(w) for w in ws], _ptr(x), fb, fe,
                                        int(threads or os.cpu_count() or 1), _ptr(y))
        if rc != 0:
            raise ValueError(f"s2o_vae_attention failed: {rc}")
        return y

    def vae_attention_tokens(self, x, weights, frame, tokens, threads=0):
        """y rows [len(tokens), C] of one frame for the selected query tokens (h*W + w)."""
        x = _f32(x)
        C, T, H, W = x.shape
        order = ["norm_bias", "norm_weight", "k_bias", "k_weight", "out_bias", "out_weight",
                 "q_bias", "q_weight", "v_bias", "v_weight"]
        ws = [_f32(weights[k]) for k in order]
        sel = np.ascontiguousarray(tokens, dtype=np.int32)
        y = np.zeros((sel.size, C), np.float32)
        rc = self.lib.s2o_vae_attention_tokens(C, T, H, W, *[_ptr(w) for w in ws], _ptr(x), int(frame),
                                               sel.ctypes.data_as(ctypes.POINTER(ctypes.c_int)), int(sel.size),
                                               int(threads or os.cpu_count() or 1), _ptr(y))
        if rc != 0:
            raise ValueError(f"s2o_vae_attention_tokens failed: {rc}")
        return y


def make_dit_input(noise, condition):
    """33-channel DiT input: noise (16) || condition (16) || ones
    (make_dit_input, src/core/engine.cpp:125-149)."""
    noise, condition = _f32(noise), _f32(condition)
    ones = np.ones((1,) + noise.shape[1:], np.float32)
    return np.concatenate([noise, condition, ones], axis=0)


def flatten_latent(latent):
    """[C, T, H, W] -> token-major [T*H*W, C] (dit.cpp:70-86)."""
    C = latent.shape[0]
    return np.ascontiguousarray(np.asarray(latent, np.float32).reshape(C, -1).T)


def unflatten_latent(flat, T, H, W):
    """token-major [T*H*W, C] -> [C, T, H, W] (dit.cpp:88-101)."""
    return np.ascontiguousarray(np.asarray(flat, np.float32).T.reshape(-1, T, H, W))


def euler_endpoint(prediction, current, timestep):
    """EulerSampler::endpoint (sampler.cpp:276-286): x - (t / 1000) * pred in fp32."""
    bt = np.float32(timestep) / np.float32(1000.0)
    return (_f32(current) - bt * _f32(prediction)).astype(np.float32)


class Ref(_Lib):
    """The reference's own CPU code (``oracle/_ref/libs2ref.so``)."""

    def __init__(self, path: str = REF_SO):
        super().__init__(path)
        L = self.lib
        L.ref_make_windows.restype = ctypes.c_int
        L.ref_make_windows.argtypes = [ctypes.c_int] * 4 + [_i32p, ctypes.c_int]
        L.ref_attention.restype = ctypes.c_int
        L.ref_attention.argtypes = (
            [_f32p, ctypes.c_int, _f32p, ctypes.c_int] + [ctypes.c_int] * 6 + [ctypes.c_float]
            + [_f32p] * 5 + [ctypes.c_int, ctypes.c_int] + [_f32p] * 6 + [_i32p])
        L.ref_block_forward.restype = ctypes.c_int
        L.ref_block_forward.argtypes = (
            [ctypes.c_int] * 8 + [ctypes.c_float, _f32p, ctypes.c_size_t, _f32p, ctypes.c_int,
                                  _f32p, ctypes.c_int, _f32p] + [ctypes.c_int] * 4 + [_f32p, _f32p])
        L.ref_vae_attention.restype = ctypes.c_int
        L.ref_vae_attention.argtypes = [ctypes.c_int] * 4 + [_f32p, ctypes.c_size_t, _f32p,
                                                              ctypes.c_int, _f32p]
        L.ref_dit_input.restype = ctypes.c_int
        L.ref_dit_input.argtypes = ([ctypes.c_int] * 5 + [_f32p, ctypes.c_size_t, _f32p] + [ctypes.c_int] * 3
                                    + [_f32p, ctypes.c_int, ctypes.c_float, ctypes.c_int] + [_f32p] * 3)
        L.ref_dit_output.restype = ctypes.c_int
        L.ref_dit_output.argtypes = ([ctypes.c_int] * 2 + [ctypes.c_float, _f32p, ctypes.c_size_t, _f32p]
                                     + [ctypes.c_int] * 3 + [_f32p, ctypes.c_int, _f32p])

    def make_windows(self, T, H, W, shifted):
        n = self.lib.ref_make_windows(T, H, W, int(shifted), None, 0)
        out = np.zeros((max(n, 1), 6), dtype=np.int32)
        self.lib.ref_make_windows(T, H, W, int(shifted), _ptr(out, _i32p), n)
        return out[:n]

    def attention(self, vid_qkv, txt_qkv, shape, heads, gammas, freqs, shifted, eps=1e-5,
                  head_count=0, threads=0, packed=False):
        T, H, W = shape
        vid_qkv, txt_qkv = _f32(vid_qkv), _f32(txt_qkv)
        L, Lt = vid_qkv.shape[0], txt_qkv.shape[0]
        dim = heads * HEAD_DIM
        vo = np.zeros((L, dim), np.float32)
        to = np.zeros((Lt, dim), np.float32)
        pk = None
        rows = ctypes.c_int(0)
        if packed:
            wins = self.make_windows(T, H, W, shifted)
            n = int(sum((w[1] - w[0]) * (w[3] - w[2]) * (w[5] - w[4]) + Lt for w in wins))
            pk = {k: np.zeros((n, dim), np.float32) for k in "qkvo"}
        g = [_f32(x) for x in gammas]
        rc = self.lib.ref_attention(
            _ptr(vid_qkv), L, _ptr(txt_qkv), Lt, T, H, W, heads, HEAD_DIM, int(shifted),
            ctypes.c_float(eps), *[_ptr(x) for x in g], _ptr(_f32(freqs)),
            int(threads or os.cpu_count() or 1), int(head_count), _ptr(vo), _ptr(to),
            *([_ptr(pk[k]) for k in "qkvo"] if pk else [None] * 4), ctypes.byref(rows))
        if rc != 0:
            raise ValueError(f"ref_attention failed: {rc}")
        return vo, to, pk

    def block_forward(self, params, weights, vid, txt, emb, shape, threads=0):
        p = params
        weights = _f32(weights)
        vid, txt, emb = _f32(vid), _f32(txt), _f32(emb)
        vo = np.zeros((vid.shape[0], p["dim"]), np.float32)
        to = np.zeros((txt.shape[0], p["dim"]), np.float32)
        rc = self.lib.ref_block_forward(
            p["block_index"], int(p["shared"]), int(p["last"]), int(p["shifted"]), p["dim"],
            p["heads"], p["head_dim"], p["mlp_hidden"], ctypes.c_float(p.get("eps", 1e-5)),
            _ptr(weights), weights.size, _ptr(vid), vid.shape[0], _ptr(txt), txt.shape[0],
            _ptr(emb), *shape, int(threads or os.cpu_count() or 1), _ptr(vo), _ptr(to))
        if rc != 0:
            raise ValueError(f"ref_block_forward failed: {rc}")
        return vo, to

    def block_forward_debug(self, params, weights, vid, txt, emb, shape, threads=0):
        """block_forward with the reference's debug capture (set_debug_tensors,
        seedvr2_dit_block.h:20-36): returns (vid_out, txt_out, {name: array})
        with the 14 capture points in SeedVR2DiTBlockDebugTensors order."""
        p = params
        weights, vid, txt, emb = _f32(weights), _f32(vid), _f32(txt), _f32(emb)
        L, Lt, d = vid.shape[0], txt.shape[0], p["dim"]
        T, H, W = shape
        wins = self.make_windows(T, H, W, p["shifted"])
        rows = int(sum((w[1] - w[0]) * (w[3] - w[2]) * (w[5] - w[4]) + Lt for w in wins))
        shapes = [(L, 3 * d), (Lt, 3 * d), (L, d), (Lt, d), (L, d), (Lt, d), (rows, d), (rows, d), (rows, d),
                  (rows, d), (L, d), (Lt, d), (L, d), (Lt, d)]
        names = ["qkv_vid", "qkv_txt", "norm_q_vid", "norm_q_txt", "norm_k_vid", "norm_k_txt", "attention_q",
                 "attention_k", "attention_v", "attention_output", "projected_vid", "projected_txt", "output_vid",
                 "output_txt"]
        caps = [np.zeros(sh, np.float32) for sh in shapes]
        arr = (_f32p * 14)(*[_ptr(c) for c in caps])
        vo = np.zeros((L, d), np.float32)
        to = np.zeros((Lt, d), np.float32)
        fn = self.lib.ref_block_forward_debug
        fn.restype = ctypes.c_int
        fn.argtypes = (self.lib.ref_block_forward.argtypes + [ctypes.POINTER(_f32p), _i32p])
        n_rows = ctypes.c_int(0)
        rc = fn(p["block_index"], int(p["shared"]), int(p["last"]), int(p["shifted"]), d, p["heads"], p["head_dim"],
                p["mlp_hidden"], ctypes.c_float(p.get("eps", 1e-5)), _ptr(weights), weights.size, _ptr(vid), L,
                _ptr(txt), Lt, _ptr(emb), T, H, W, int(threads or os.cpu_count() or 1), _ptr(vo), _ptr(to), arr,
                ctypes.byref(n_rows))
        if rc != 0:
            raise ValueError(f"ref_block_forward_debug failed: {rc}")
        assert n_rows.value == rows
        return vo, to, dict(zip(names, caps))

    def dit_input(self, params, weights, latent33, text, timestep, threads=0):
        """SeedVR2DiTInput on latent [vc, T, H, W] (flattened here like
        SeedVR2DiT::forward, dit.cpp:70-86, 298) and text [Lt, tc].
        Returns (vid [T*H/2*W/2, dim], txt [Lt, dim], emb [ed])."""
        p = params
        latent33, text, weights = _f32(latent33), _f32(text), _f32(weights)
        vc, T, H, W = latent33.shape
        flat = np.ascontiguousarray(flatten_latent(latent33))
        rows = T * (H // 2) * (W // 2)
        vo = np.zeros((rows, p["dim"]), np.float32)
        to = np.zeros((text.shape[0], p["dim"]), np.float32)
        emb = np.zeros(p["embedding_dim"], np.float32)
        rc = self.lib.ref_dit_input(p["dim"], vc, p["text_channels"], p["sinusoidal_dim"], p["embedding_dim"],
                                    _ptr(weights), weights.size, _ptr(flat), T, H, W, _ptr(text), text.shape[0],
                                    ctypes.c_float(timestep), int(threads or os.cpu_count() or 1), _ptr(vo),
                                    _ptr(to), _ptr(emb))
        if rc != 0:
            raise ValueError(f"ref_dit_input failed: {rc}")
        return vo, to, emb

    def dit_output(self, params, weights, vid, emb, patched_shape, threads=0):
        """SeedVR2DiTOutput; returns the prediction [oc, T, 2H, 2W] (unflattened
        like dit.cpp:88-101)."""
        p = params
        vid, emb, weights = _f32(vid), _f32(emb), _f32(weights)
        T, H, W = patched_shape
        oc = p["out_channels"]
        flat = np.zeros((T * 2 * H * 2 * W, oc), np.float32)
        rc = self.lib.ref_dit_output(p["dim"], oc, ctypes.c_float(p.get("eps", 1e-5)), _ptr(weights), weights.size,
                                     _ptr(vid), T, H, W, _ptr(emb), int(threads or os.cpu_count() or 1), _ptr(flat))
        if rc != 0:
            raise ValueError(f"ref_dit_output failed: {rc}")
        return unflatten_latent(flat, T, 2 * H, 2 * W)

    def euler_step(self, head_params, input_weights, block_params, block_weights, output_weights, noise, condition,
                   text, timestep=1000.0, threads=0):
        """One DiT Euler step the way the reference engine runs it with one
        sampling step and cfg 1 (engine.cpp:308-343): make_dit_input, the DiT
        forward (input head, blocks in order, output head; dit.cpp:277-383)
        and EulerSampler::endpoint (sampler.cpp:276-286)."""
        latent = make_dit_input(noise, condition)
        vid, txt, emb = self.dit_input(head_params, input_weights, latent, text, timestep, threads)
        _, T, H, W = latent.shape
        shape = (T, H // 2, W // 2)
        for bp, bw in zip(block_params, block_weights):
            vid, txt = self.block_forward(bp, bw, vid, txt, emb, shape, threads)
        pred = self.dit_output(head_params, output_weights, vid, emb, shape, threads)
        return euler_endpoint(pred, noise, timestep), pred

    def sample(self, head_params, input_weights, block_params, block_weights, output_weights, noise, condition,
               positive_text, negative_text=None, steps=1, cfg_scale=1.0, cfg_rescale=0.0, threads=0):
        """The engine's sampling loop (engine.cpp:308-347) on the reference's
        own code: make_dit_input (restated), the DiT forward layer by layer,
        and EulerSampler (apply_cfg, step_to, endpoint) from sampler.cpp."""
        s = SamplerRef(self.lib)
        ts = s.timesteps(steps)
        latent = _f32(noise)
        _, T, H, W = latent.shape
        shape = (T, H // 2, W // 2)

        def predict(text, t):
            vid, txt, emb = self.dit_input(head_params, input_weights, make_dit_input(latent, condition), text, t,
                                           threads)
            for bp, bw in zip(block_params, block_weights):
                vid, txt = self.block_forward(bp, bw, vid, txt, emb, shape, threads)
            return self.dit_output(head_params, output_weights, vid, emb, shape, threads)

        for i, t in enumerate(ts):
            pred = predict(positive_text, float(t))
            if cfg_scale != 1.0:
                pred = s.apply_cfg(pred, predict(negative_text, float(t)), cfg_scale, cfg_rescale)
            latent = s.step_to(pred, latent, float(t), float(ts[i + 1])) if i + 1 < len(ts) else \
                s.endpoint(pred, latent, float(t))
        return latent

    def group_norm(self, x, bias, weight, threads=0):
        """The reference's DynamicFramewiseGroupNorm on x [C, T, H, W]."""
        x = _f32(x)
        C, T, H, W = x.shape
        y = np.zeros_like(x)
        L = self.lib
        L.ref_group_norm.restype = ctypes.c_int
        L.ref_group_norm.argtypes = [ctypes.c_int] * 4 + [_f32p] * 3 + [ctypes.c_int, _f32p]
        rc = L.ref_group_norm(C, T, H, W, _ptr(_f32(bias)), _ptr(_f32(weight)), _ptr(x),
                              int(threads or os.cpu_count() or 1), _ptr(y))
        if rc != 0:
            raise ValueError(f"ref_group_norm failed: {rc}")
        return y

    def space_time_shuffle(self, x, bias, weight, threads=0):
        """The reference's DynamicSpaceTimeShuffle: x [Cin, T, H, W], weight [P, Cin]."""
        x = _f32(x)
        C, T, H, W = x.shape
        P = int(np.asarray(bias).size)
        L = self.lib
        L.ref_space_time_shuffle.restype = ctypes.c_int
        L.ref_space_time_shuffle.argtypes = [ctypes.c_int] * 5 + [_f32p] * 3 + [ctypes.c_int, _f32p, _i32p]
        of = ctypes.c_int(0)
        tr = P // C // 4
        y = np.zeros((C, T * tr - 1 if tr > 1 else T, 2 * H, 2 * W), np.float32)
        rc = L.ref_space_time_shuffle(C, P, T, H, W, _ptr(_f32(bias)), _ptr(_f32(weight)), _ptr(x),
                                      int(threads or os.cpu_count() or 1), _ptr(y), ctypes.byref(of))
        if rc != 0:
            raise ValueError(f"ref_space_time_shuffle failed: {rc}")
        assert of.value == y.shape[1]
        return y

    def vae_attention(self, x, weights_flat, threads=0):
        x = _f32(x)
        C, T, H, W = x.shape
        w = _f32(weights_flat)
        y = np.zeros_like(x)
        rc = self.lib.ref_vae_attention(C, T, H, W, _ptr(w), w.size, _ptr(x),
                                        int(threads or os.cpu_count() or 1), _ptr(y))
        if rc != 0:
            raise ValueError(f"ref_vae_attention failed: {rc}")
        return y


def _sampler_port_init(L):
    L.s2o_sampler_timesteps.restype = None
    L.s2o_sampler_timesteps.argtypes = [ctypes.c_int, _f32p]
    L.s2o_apply_cfg.restype = None
    L.s2o_apply_cfg.argtypes = [_f32p, _f32p, ctypes.c_size_t, ctypes.c_float, ctypes.c_float, _f32p]
    L.s2o_euler_step_to.restype = None
    L.s2o_euler_step_to.argtypes = [_f32p, _f32p, ctypes.c_size_t, ctypes.c_float, ctypes.c_float, _f32p]
    L.s2o_euler_endpoint.restype = None
    L.s2o_euler_endpoint.argtypes = [_f32p, _f32p, ctypes.c_size_t, ctypes.c_float, _f32p]
    L.s2o_condition_ratio.restype = ctypes.c_float
    L.s2o_condition_ratio.argtypes = [ctypes.c_float] + [ctypes.c_int] * 3
    L.s2o_make_condition.restype = None
    L.s2o_make_condition.argtypes = [_f32p, _f32p, ctypes.c_size_t, ctypes.c_float, _f32p]


class SamplerPort:
    """EulerSampler restated in C (oracle/s2_oracle.c; sampler.cpp:19-62,
    181-286) and the condition builder (engine.cpp:79-121)."""

    def __init__(self, port_lib):
        self.lib = port_lib
        _sampler_port_init(port_lib)

    def timesteps(self, steps):
        out = np.zeros(max(int(steps), 1), np.float32)
        self.lib.s2o_sampler_timesteps(int(steps), _ptr(out))
        return out

    def apply_cfg(self, pos, neg, scale, rescale=0.0):
        pos, neg = _f32(pos), _f32(neg)
        out = np.empty_like(pos)
        self.lib.s2o_apply_cfg(_ptr(pos), _ptr(neg), pos.size, ctypes.c_float(scale), ctypes.c_float(rescale), _ptr(out))
        return out

    def step_to(self, pred, cur, t, t_next):
        pred, cur = _f32(pred), _f32(cur)
        out = np.empty_like(cur)
        self.lib.s2o_euler_step_to(_ptr(pred), _ptr(cur), cur.size, ctypes.c_float(t), ctypes.c_float(t_next), _ptr(out))
        return out

    def endpoint(self, pred, cur, t):
        pred, cur = _f32(pred), _f32(cur)
        out = np.empty_like(cur)
        self.lib.s2o_euler_endpoint(_ptr(pred), _ptr(cur), cur.size, ctypes.c_float(t), _ptr(out))
        return out

    def condition_ratio(self, noise_scale, frames, height, width):
        return float(self.lib.s2o_condition_ratio(ctypes.c_float(noise_scale), frames, height, width))

    def make_condition(self, encoded, noise, noise_scale):
        encoded, noise = _f32(encoded), _f32(noise)
        _, T, H, W = encoded.shape
        out = np.empty_like(encoded)
        self.lib.s2o_make_condition(_ptr(encoded), _ptr(noise), encoded.size,
                                    ctypes.c_float(self.condition_ratio(noise_scale, T, H, W)), _ptr(out))
        return out


class SamplerRef:
    """The reference's own EulerSampler (src/model/sampler.cpp, compiled into
    oracle/_ref/libs2ref.so by oracle/ref_sampler.cpp)."""

    def __init__(self, ref_lib):
        L = self.lib = ref_lib
        L.ref_sampler_timesteps.restype = ctypes.c_int
        L.ref_sampler_timesteps.argtypes = [ctypes.c_int, _f32p]
        L.ref_apply_cfg.restype = ctypes.c_int
        L.ref_apply_cfg.argtypes = [_f32p, _f32p] + [ctypes.c_int] * 4 + [ctypes.c_float, ctypes.c_float, _f32p]
        L.ref_step_to.restype = ctypes.c_int
        L.ref_step_to.argtypes = [_f32p, _f32p] + [ctypes.c_int] * 4 + [ctypes.c_float, ctypes.c_float, _f32p]
        L.ref_endpoint.restype = ctypes.c_int
        L.ref_endpoint.argtypes = [_f32p, _f32p] + [ctypes.c_int] * 4 + [ctypes.c_float, _f32p]

    def timesteps(self, steps):
        out = np.zeros(max(int(steps), 1), np.float32)
        n = self.lib.ref_sampler_timesteps(int(steps), _ptr(out))
        return out[:n]

    def apply_cfg(self, pos, neg, scale, rescale=0.0):
        pos, neg = _f32(pos), _f32(neg)
        out = np.empty_like(pos)
        rc = self.lib.ref_apply_cfg(_ptr(pos), _ptr(neg), *pos.shape, ctypes.c_float(scale), ctypes.c_float(rescale),
                                    _ptr(out))
        if rc != 0:
            raise ValueError(f"ref_apply_cfg failed: {rc}")
        return out

    def step_to(self, pred, cur, t, t_next):
        pred, cur = _f32(pred), _f32(cur)
        out = np.empty_like(cur)
        rc = self.lib.ref_step_to(_ptr(pred), _ptr(cur), *cur.shape, ctypes.c_float(t), ctypes.c_float(t_next), _ptr(out))
        if rc != 0:
            raise ValueError(f"ref_step_to failed: {rc}")
        return out

    def endpoint(self, pred, cur, t):
        pred, cur = _f32(pred), _f32(cur)
        out = np.empty_like(cur)
        rc = self.lib.ref_endpoint(_ptr(pred), _ptr(cur), *cur.shape, ctypes.c_float(t), _ptr(out))
        if rc != 0:
            raise ValueError(f"ref_endpoint failed: {rc}")
        return out


def port() -> Port:
    return Port()


def ref() -> Ref | None:
    return Ref() if os.path.exists(REF_SO) else None
