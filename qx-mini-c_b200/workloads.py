"""Seeded synthetic workloads for the five BASELINE configurations.

No dataset or checkpoint exists here, so every input is generated from a seed:
the model by qxh_synth_build (libqxhost.so) and the activations / KV history
by qxh_normal_vector.  Tests, the golden-fixture script and bench.py all build
their inputs through these functions, so the engine and the CPU checkers see
identical bytes.
"""
import numpy as np

import qxlib

MODEL_SEED = 7
START_TOKEN = 42          # config 4: greedy decode from token 42
DECODE_STEPS = 256        # config 4: 256 greedy steps
HEAD_X_SEED = 1           # config 1: x ~ N(0,1), RMSNorm-ed with unit weight inside the head
MOE_LAYER = 3             # config 2: one MoE layer, hidden ~ N(0,1)
MOE_X_SEED = 1
ATTN_LAYER = 5            # config 3: one attention layer with N(0,1) INT8 history
ATTN_X_SEED = 3
ATTN_HISTORY_SEED = 11


def model_config(full=True, seed=MODEL_SEED):
    return qxlib.synth_config(seed) if full else qxlib.mini_config(seed)


def head_input(hidden):
    return qxlib.normal_vector(HEAD_X_SEED, hidden)


def moe_input(hidden):
    return qxlib.normal_vector(MOE_X_SEED, hidden)


def attn_input(hidden):
    return qxlib.normal_vector(ATTN_X_SEED, hidden)


def attn_history(positions, kv_values, quantize):
    """N(0,1) K and V vectors for `positions` tokens, quantized one token at a
    time with `quantize(vec) -> (int8[kv_values], scale)` (the reference's
    per-token INT8 rule).  Returns k, v int8 [positions][kv_values] and scales."""
    raw = qxlib.normal_vector(ATTN_HISTORY_SEED, 2 * positions * kv_values).reshape(positions, 2, kv_values)
    k = np.zeros((positions, kv_values), np.int8)
    v = np.zeros((positions, kv_values), np.int8)
    ks = np.zeros(positions, np.float32)
    vs = np.zeros(positions, np.float32)
    for t in range(positions):
        k[t], ks[t] = quantize(raw[t, 0])
        v[t], vs[t] = quantize(raw[t, 1])
    return k, v, ks, vs


def weight_bytes_per_token(cfg):
    """Algorithmic HBM bytes one batch-1 decode step must read: every
    attention/router weight of every layer, the 8 selected experts' gate/up/
    down slices, the embedding row, both norms and the whole head."""
    H, L, E, I = cfg.hidden, cfg.layers, cfg.experts, cfg.moe_intermediate
    Q, KV, V = cfg.q_heads * cfg.head_dim, cfg.kv_heads * cfg.head_dim, cfg.vocab
    iq4 = lambda rows, k: rows * (k // 256) * 136
    iq2 = lambda rows, k: rows * (k // 256) * 74
    iq3 = lambda rows, k: rows * (k // 256) * 98
    per_layer = (iq4(Q, H) + 2 * iq4(KV, H) + iq4(H, Q) + E * H * 4 + 8 * (2 * iq2(I, H) + iq3(H, I))
                 + 4 * (2 * H + 2 * cfg.head_dim))
    return L * per_layer + (H // 256) * 144 + H * 4 + V * (H // 256) * 210


def kv_bytes_per_token(cfg, position):
    """INT8 K+V plus two scales per layer for positions 0..position."""
    KV = cfg.kv_heads * cfg.head_dim
    return cfg.layers * (position + 1) * (2 * KV + 8)
