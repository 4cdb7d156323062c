"""The oracle's decode step (oracle/cpu_decoder.c, cd_step) set up for a device decoder — TEST
INFRASTRUCTURE ONLY, used by the decoder parity tests and by the smoke entry point.

The weights are generated on the device; the checker rebuilds them on the host: the expert
banks bit for bit from the same seeds (the integer generator is identical on both sides), the
bf16 projections by unpacking the packed tiles, the f32 tensors by download. The checker keeps
its own KV pools (zeroed), indexed through the device's page tables.
"""
import ctypes as C

import numpy as np

import oracle as O
from moearc_b200.decoder import Decoder, unpack_dense


def host_model(dec: Decoder):
    cfg = dec.cfg
    H, Dq, Dkv = cfg.n_embd, cfg.n_head * cfg.head_dim, cfg.n_head_kv * cfg.head_dim
    nb = cfg.n_expert * cfg.n_ff * H // 32
    layers, keep = [], []
    for l in range(cfg.n_layer):
        t = {}
        t["attn_norm"] = dec.tensor(0, l, np.float32)
        t["ffn_norm"] = dec.tensor(1, l, np.float32)
        t["sinks"] = dec.tensor(2, l, np.float32) if cfg.has_sinks else None
        t["router"] = dec.tensor(3, l, np.float32)
        wqkv = unpack_dense(dec.tensor(7, l, np.uint16), Dq + 2 * Dkv, H)
        t["wq"] = np.ascontiguousarray(wqkv[:Dq])
        t["wk"] = np.ascontiguousarray(wqkv[Dq:Dq + Dkv])
        t["wv"] = np.ascontiguousarray(wqkv[Dq + Dkv:])
        t["wo"] = np.ascontiguousarray(unpack_dense(dec.tensor(8, l, np.uint16), H, Dq))
        synth = O.synth_mxfp4 if cfg.expert_type == O.MXFP4 else (lambda s, n: O.synth_q4_0(s, n, 0.01))
        t["gate"], t["up"], t["down"] = (synth(dec.seed(k, l), nb) for k in (8, 9, 10))
        kp = dec.tensor(4, l, np.uint16)
        t["k"], t["v"] = np.zeros_like(kp), np.zeros_like(kp)
        t["table"] = dec.tensor(6, l, np.uint32)
        t["q_norm"] = dec.tensor(15, l, np.float32) if cfg.has_qk_norm else None
        t["k_norm"] = dec.tensor(16, l, np.float32) if cfg.has_qk_norm else None
        keep.append(t)
        layers.append(O.CdLayer(*[O.ptr(t[n]) if t[n] is not None else None for n in
                                  ("attn_norm", "ffn_norm", "wq", "wk", "wv", "wo", "sinks", "router",
                                   "gate", "up", "down", "k", "v", "table", "q_norm", "k_norm")]))
    arr = (O.CdLayer * cfg.n_layer)(*layers)
    c = O.CdCfg(cfg.n_layer, H, cfg.n_head, cfg.n_head_kv, cfg.head_dim, cfg.n_expert, cfg.n_ff,
                cfg.n_expert_used, cfg.gating, cfg.act, cfg.expert_type, O.BF16, cfg.alpha, cfg.limit,
                cfg.rms_eps, cfg.n_swa, cfg.swa_pattern, 32, cfg.rope_base, cfg.rope_freq_scale,
                cfg.rope_ext_factor, cfg.rope_attn_factor, cfg.rope_corr_lo, cfg.rope_corr_hi, cfg.has_qk_norm)
    return c, arr, keep, dec.tensor(11, 0, np.float32)


def oracle_step(c, arr, out_norm, x, pos):
    want = np.zeros(c.n_embd, np.float32)
    assert O.lib().cd_step(C.byref(c), arr, O.ptr(out_norm), O.ptr(x), pos, None, O.ptr(want), None) == 0
    return want


def rel_to_oracle(got, want):
    return float(np.max(np.abs(got.astype(np.float64) - want) / np.maximum(np.abs(want), 1.0)))


def oracle_logits(c, dec: Decoder, x_normed):
    """The output head on the oracle's normalised final state (cd_logits), from the decoder's
    packed head weights unpacked to rows."""
    w = np.ascontiguousarray(unpack_dense(dec.tensor(17, 0, np.uint16), dec.cfg.n_vocab, dec.cfg.n_embd))
    out = np.zeros(dec.cfg.n_vocab, np.float32)
    x = np.ascontiguousarray(x_normed, np.float32)
    assert O.lib().cd_logits(C.byref(c), O.ptr(w), dec.cfg.n_vocab, O.ptr(x), O.ptr(out)) == 0
    return out
