"""CPU restatement of the reference decoder step -- TEST INFRASTRUCTURE ONLY.

numpy (fp32) restatement of qkn_decoder_prefill (qkn_decoder.c:369-564) and
qkn_decoder_forward (qkn_decoder.c:570-714) in the configurations the device decoder
step implements: Qwen3 (per-head QK-RMSNorm, NeoX RoPE, SwiGLU, residual then norm)
and Gemma (the exports' settings, paligemma.c:206-230: embedding scale, interleaved
RoPE, GeGLU, a norm on each sublayer's output before its residual add
(qkn_decoder.c:681-704), attention softcap, sliding-window layers with their own
RoPE theta, QK-norm optional); interleaved gate/up rows, tied embeddings, greedy argmax.
The attention, QK-norm, RoPE and cache append go through the C restatement
(pyoracle: smol_oracle.c) over a cache that holds the device formats (K bf16, V
fp16), so both sides attend over identical values.  Weights are bf16 (kept as the
rounded fp32 values and as the raw bits to upload).

Pinned to the reference decoder itself: PIN_CASES below run through qkn_decoder.c (and
SmolVLM's decoder.c) on the same weights, live in tests/test_decoder_oracle_e2e.py and
as the committed outputs of tests/golden/decoder_cases.npz; its pieces are pinned to the
reference's own kernels in tests/test_decoder_oracle.py.

Only tests/ import this module.
"""
from __future__ import annotations

import struct

import numpy as np

import pyoracle


def rms_norm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """smol_rms_norm (rmsnorm.c:17-70): (x * w) * 1/sqrtf(mean(x^2) + eps), per row."""
    ss = np.sum(x.astype(np.float32) ** 2, axis=-1, keepdims=True, dtype=np.float32)
    inv = (np.float32(1.0) / np.sqrt(ss / np.float32(x.shape[-1]) + np.float32(eps))).astype(np.float32)
    return ((x * w).astype(np.float32) * inv).astype(np.float32)


def swiglu(gate_up: np.ndarray) -> np.ndarray:
    """smol_swiglu_multiply (activation.c:55-86): silu(g[2j]) * g[2j+1]."""
    g = gate_up[..., 0::2]
    u = gate_up[..., 1::2]
    return ((g / (np.float32(1.0) + np.exp(-g, dtype=np.float32))) * u).astype(np.float32)


def geglu(gate_up: np.ndarray) -> np.ndarray:
    """smol_geglu_multiply (activation.c:104-126): gelu_tanh(g[2j]) * g[2j+1]."""
    g = gate_up[..., 0::2]
    u = gate_up[..., 1::2]
    x3 = (g * g * g).astype(np.float32)
    inner = (np.float32(0.7978845608028654) * (g + np.float32(0.044715) * x3)).astype(np.float32)
    gl = (np.float32(0.5) * g * (np.float32(1.0) + np.tanh(inner, dtype=np.float32))).astype(np.float32)
    return (gl * u).astype(np.float32)


def argmax_first(logits: np.ndarray) -> int:
    """smol_argmax_matvec_bf16 (matmul.c:392-417): the lowest index among equal maxima."""
    return int(np.argmax(logits))


class QknOracle:
    """A seeded decoder (Qwen3 or Gemma configuration) and its reference forward passes."""

    def __init__(self, hidden=1024, layers=2, n_heads=16, n_kv_heads=8, head_dim=128, intermediate=3072,
                 vocab=4096, theta=1e6, eps=1e-6, qk_gain=3.0, vo_gain=4.0, seed=0, cap=1024, gemma=None,
                 qk_norm=True, tied=True):
        """gemma (None for Qwen3): dict of the Gemma settings -- embed_normalizer, attn_softcap,
        sliding_window, sliding (per-layer flags), local_theta, qk_norm (bool), interleaved (bool),
        sublayer_gain.  Gemma models carry pre/post-FFN norms and use GeGLU.
        qk_norm=False, tied=False: SmolVLM's decoder (exports/smolvlm/decoder.c:391-476) --
        no per-head QK-norm, an lm_head of its own."""
        rng = np.random.default_rng(seed)
        self.H, self.L, self.HQ, self.HKV, self.HD = hidden, layers, n_heads, n_kv_heads, head_dim
        self.I, self.V, self.eps, self.cap = intermediate, vocab, eps, cap
        self.theta = theta
        g = dict(gemma or {})
        self.gemma = gemma is not None
        self.embed_normalizer = np.float32(g.get("embed_normalizer", 0.0))
        self.attn_softcap = float(g.get("attn_softcap", 0.0))
        self.sliding_window = int(g.get("sliding_window", 0))
        self.sliding = [bool(x) for x in g.get("sliding", [False] * layers)]
        self.local_theta = float(g.get("local_theta", 0.0))
        self.qk_norm = bool(g.get("qk_norm", qk_norm))
        self.interleaved = bool(g.get("interleaved", False))
        qd, kvd = n_heads * head_dim, n_kv_heads * head_dim

        def bf(*shape, sc=1.0):
            return pyoracle.round_bf16((rng.standard_normal(shape) * sc).astype(np.float32))

        def near(n, mean, sd=0.02):
            return (mean + sd * rng.standard_normal(n)).astype(np.float32)

        # Gemma's embedding rows are small and scaled up by embed_normalizer on lookup
        self.E = bf(vocab, hidden, sc=1 / float(self.embed_normalizer) if self.embed_normalizer > 0 else 1.0)
        self.final_norm = near(hidden, 1.0)
        self.layers = []
        for _ in range(layers):
            self.layers.append({
                "wq": bf(qd, hidden, sc=1 / np.sqrt(hidden)),
                "wk": bf(kvd, hidden, sc=1 / np.sqrt(hidden)),
                "wv": bf(kvd, hidden, sc=vo_gain / np.sqrt(hidden)),
                "wo": bf(hidden, qd, sc=vo_gain / np.sqrt(qd)),
                "gate_up": bf(2 * intermediate, hidden, sc=1 / np.sqrt(hidden)),
                "down": bf(hidden, intermediate, sc=1 / np.sqrt(intermediate)),
                "input_norm": near(hidden, 1.0),
                "post_attn_norm": near(hidden, 1.0),
                "q_norm": near(head_dim, qk_gain),
                "k_norm": near(head_dim, qk_gain),
            })
            if not self.gemma and not self.qk_norm:
                del self.layers[-1]["q_norm"], self.layers[-1]["k_norm"]
            if self.gemma:
                # the sublayer-output norms scale each sublayer's contribution against the
                # embedding (sublayer_gain, so that the next token is not the fed one)
                gain = np.float32(g.get("sublayer_gain", 4.0))
                self.layers[-1]["post_attn_norm"] = (self.layers[-1]["post_attn_norm"] * gain).astype(np.float32)
                self.layers[-1]["pre_ffn_norm"] = near(hidden, 1.0)
                self.layers[-1]["post_ffn_norm"] = (near(hidden, 1.0) * gain).astype(np.float32)
                if not self.qk_norm:
                    del self.layers[-1]["q_norm"], self.layers[-1]["k_norm"]
        # an untied output head is drawn last, so the tied models' weights do not move
        self.lm_head = None if tied else bf(vocab, hidden)
        self.cos, self.sin = pyoracle.fill_rope_table(cap, head_dim, theta, self.interleaved)
        # sliding layers use their own table when the theta differs (qkn_decoder.c:313-340, :462-468)
        self.has_local = self.local_theta > 0 and self.local_theta != theta
        if self.has_local:
            self.cos_local, self.sin_local = pyoracle.fill_rope_table(cap, head_dim, self.local_theta, self.interleaved)
        self.kc = [np.zeros((cap, kvd), np.uint16) for _ in range(layers)]   # bf16 bits
        self.vc = [np.zeros((cap, kvd), np.uint16) for _ in range(layers)]   # fp16 bits
        self.len = 0
        self.o = pyoracle.oracle()
        self.scale = np.float32(1.0 / np.sqrt(np.float32(head_dim)))

    def _layer(self, l: int, x: np.ndarray, pos0: int, device_formats: bool = False) -> np.ndarray:
        """One decoder layer over tokens at positions pos0.. (qkn_decoder.c:431-563 / :622-705).
        device_formats: round what the device prefill keeps in bf16 -- the RMSNorm outputs,
        the rotated Q, the attention output and the gated activation (GEMM / attention
        operands) -- the same way; the Q / K / V projections take the input RMSNorm output
        as two bf16 operands, hi = bf16(x) and lo = bf16(x - hi), summed in fp32."""
        r16 = pyoracle.round_bf16 if device_formats else (lambda a: a)
        lw, n = self.layers[l], x.shape[0]
        sliding = self.sliding[l] and self.sliding_window > 0
        cos, sin = (self.cos_local, self.sin_local) if self.has_local and self.sliding[l] else (self.cos, self.sin)
        xn = rms_norm(x, lw["input_norm"], self.eps)
        if device_formats:
            hi = r16(xn)
            lo = r16((xn - hi).astype(np.float32))
            q, k, v = ((hi @ lw[w].T).astype(np.float32) + (lo @ lw[w].T).astype(np.float32) for w in ("wq", "wk", "wv"))
        else:
            q, k, v = xn @ lw["wq"].T, xn @ lw["wk"].T, xn @ lw["wv"].T
        pos = np.arange(pos0, pos0 + n, dtype=np.int32)
        q_rot = pyoracle.qknorm_rope_append(q, k, v, self.HQ, self.HKV, self.HD, lw.get("q_norm"), lw.get("k_norm"),
                                            self.eps, cos, sin, self.interleaved, pos, pos.astype(np.int64),
                                            self.kc[l], self.vc[l])
        total = pos0 + n
        K = pyoracle.bf16_to_f32(self.kc[l][:total])
        Vv = self.vc[l][:total].view(np.float16).astype(np.float32)
        attn = self.o.causal_attention(r16(q_rot), K, Vv, n, total, self.HQ, self.HKV, self.HD, self.scale, pos0,
                                       window=self.sliding_window if sliding else 0, cap=self.attn_softcap)
        proj = (r16(attn) @ lw["wo"].T).astype(np.float32)
        if "pre_ffn_norm" in lw:   # Gemma: norm the sublayer output, add, norm for the MLP (:681-685)
            x = (x + rms_norm(proj, lw["post_attn_norm"], self.eps)).astype(np.float32)
            xn = r16(rms_norm(x, lw["pre_ffn_norm"], self.eps))
        else:                      # Qwen3: add, then norm (:688-689)
            x = (x + proj).astype(np.float32)
            xn = r16(rms_norm(x, lw["post_attn_norm"], self.eps))
        gu = xn @ lw["gate_up"].T
        act = r16(geglu(gu) if self.gemma else swiglu(gu))
        ffn = (act @ lw["down"].T).astype(np.float32)
        if "post_ffn_norm" in lw:
            ffn = rms_norm(ffn, lw["post_ffn_norm"], self.eps)
        return (x + ffn).astype(np.float32)

    def _embed(self, tokens) -> np.ndarray:
        """Embedding rows, scaled by embed_normalizer when it is set (qkn_decoder.c:415-419, :596-599)."""
        x = self.E[np.asarray(tokens)].astype(np.float32)
        if self.embed_normalizer > 0:
            x = (x * self.embed_normalizer).astype(np.float32)
        return x

    def prefill(self, tokens, device_formats: bool = False) -> None:
        """qkn_decoder_prefill over `tokens` (no logits, as the reference); device_formats:
        the operand roundings of the device prefill (smol_b200_qkn_prefill)."""
        x = self._embed(tokens)
        for l in range(self.L):
            x = self._layer(l, x, self.len, device_formats)
        self.len += len(tokens)

    def forward(self, token: int) -> tuple[int, float, np.ndarray]:
        """qkn_decoder_forward for one token: (greedy token, top-1/top-2 margin, final normed x)."""
        x = self._embed([token])
        for l in range(self.L):
            x = self._layer(l, x, self.len)
        self.len += 1
        xf = rms_norm(x, self.final_norm, self.eps)[0]
        logits = (self.E if self.lm_head is None else self.lm_head) @ xf
        top = np.argsort(logits)[-2:]
        return argmax_first(logits), float(logits[top[1]] - logits[top[0]]), xf

    def device_weights(self, to_device):
        """Upload helper: to_device(np array) -> device tensor; bf16 matrices go as raw bits."""
        bits = lambda a: to_device(pyoracle.bf16_bits(a))   # noqa: E731
        layers = [{name: (bits(w) if w.ndim == 2 else to_device(w)) for name, w in lw.items()} for lw in self.layers]
        return bits(self.E), to_device(self.final_norm), layers


# ---------------------------------------------------------------------------
# Cases that pin this restatement to the reference decoder (qkn_decoder.c run on the
# same weights by oracle/_ref/qkn_weights_emul, built from tests/dropin/qkn_weights_main.c)
# ---------------------------------------------------------------------------
# Gemma settings as the exports set them (paligemma.c:206-230), at test scale: Gemma 2
# (no QK-norm, attention softcap, alternating sliding layers with their own RoPE theta)
# and Gemma 3 (QK-norm, no softcap); the window is short enough to bind.
GEMMA2_SMALL = {"embed_normalizer": 32.0, "interleaved": True, "attn_softcap": 3.0, "sliding_window": 16,
                "sliding": [True, False], "local_theta": 1e4, "qk_norm": False}
GEMMA3_SMALL = {"embed_normalizer": 32.0, "interleaved": True, "attn_softcap": 0.0, "sliding_window": 16,
                "sliding": [True, False], "local_theta": 1e4, "qk_norm": True}
GEMMA_SHAPE = {"n_heads": 8, "n_kv_heads": 1, "head_dim": 256, "intermediate": 2048}
PIN_CASES = {
    "qwen3-1": {"layers": 1, "prompt_len": 96, "steps": 24, "seed": 11, "gemma": None},
    "qwen3-2": {"layers": 2, "prompt_len": 64, "steps": 24, "seed": 12, "gemma": None},
    "gemma2-2": {"layers": 2, "prompt_len": 64, "steps": 24, "seed": 13, "gemma": GEMMA2_SMALL},
    "gemma3-2": {"layers": 2, "prompt_len": 64, "steps": 24, "seed": 14, "gemma": GEMMA3_SMALL},
    # SmolVLM's decoder (run by oracle/_ref/smolvlm_weights_ref): MHA with head dim 64,
    # no QK-norm, an untied lm_head, its RoPE theta and epsilon
    "smolvlm-2": {"layers": 2, "prompt_len": 64, "steps": 24, "seed": 15, "gemma": None, "smolvlm": True},
}
SMOLVLM_SHAPE = {"hidden": 512, "n_heads": 8, "n_kv_heads": 8, "head_dim": 64, "intermediate": 1536,
                 "theta": 273768.0, "eps": 1e-5, "qk_norm": False, "tied": False}


def pin_case(name: str):
    """(model, prompt, feed) of a pin case: the seeded model (not prefilled), its prompt,
    and the tokens fed at each teacher-forced step -- the prompt's last token, then a
    seeded random stream (random models' own greedy streams tend to settle on one token)."""
    c = PIN_CASES[name]
    shape = dict(theta=1e6, eps=1e-6)
    shape.update(GEMMA_SHAPE if c["gemma"] else (SMOLVLM_SHAPE if c.get("smolvlm") else {}))
    m = QknOracle(layers=c["layers"], seed=c["seed"], qk_gain=3.0, vo_gain=4.0,
                  cap=c["prompt_len"] + c["steps"] + 8, gemma=c["gemma"], **shape)
    rng = np.random.default_rng(c["seed"])
    prompt = rng.integers(0, m.V, c["prompt_len"]).tolist()
    feed = [prompt[-1]] + rng.integers(0, m.V, c["steps"] - 1).tolist()
    return m, prompt, feed


def run_teacher_forced(m: QknOracle, prompt, feed):
    """Prefill prompt[:-1], then one forward per fed token: (tokens, margins, final normed states)."""
    m.prefill(prompt[:-1])
    out = [m.forward(t) for t in feed]
    return [o[0] for o in out], [o[1] for o in out], np.stack([o[2] for o in out])


def write_weights_file(path, m: QknOracle, prompt, feed) -> None:
    """The input file of qkn_weights_main.c (its header comment gives the format)."""
    bits = lambda a: np.ascontiguousarray(pyoracle.bf16_bits(a)).tobytes()        # noqa: E731
    f32 = lambda a: np.ascontiguousarray(a, dtype=np.float32).tobytes()              # noqa: E731
    has_ffn_norms = int("pre_ffn_norm" in m.layers[0])
    with open(path, "wb") as f:
        f.write(b"QKNW")
        f.write(struct.pack("<14i", m.H, m.L, m.HQ, m.HKV, m.HD, m.I, m.V, len(prompt), len(feed), int(m.gemma),
                            int(m.interleaved), m.sliding_window, int(m.qk_norm), has_ffn_norms))
        f.write(struct.pack("<5f", m.eps, m.theta, m.local_theta, float(m.embed_normalizer), m.attn_softcap))
        f.write(bits(m.E))
        f.write(f32(m.final_norm))
        for l, lw in enumerate(m.layers):
            f.write(struct.pack("<i", int(m.sliding[l])))
            for name in ("wq", "wk", "wv", "wo", "gate_up", "down"):
                f.write(bits(lw[name]))
            names = ["input_norm", "post_attn_norm"] + (["q_norm", "k_norm"] if m.qk_norm else []) + \
                (["pre_ffn_norm", "post_ffn_norm"] if has_ffn_norms else [])
            for name in names:
                f.write(f32(lw[name]))
        f.write(np.asarray(prompt, "<i4").tobytes())
        f.write(np.asarray(feed, "<i4").tobytes())
        if m.lm_head is not None:   # read by the SmolVLM driver only
            f.write(bits(m.lm_head))


def read_reference_steps(path, n_steps: int, hidden: int):
    """qkn_weights_main.c's output: per step the greedy token and the final normed state."""
    raw = np.fromfile(path, dtype=np.uint8).reshape(n_steps, 4 + 4 * hidden)
    return raw[:, :4].copy().view("<i4")[:, 0], raw[:, 4:].copy().view("<f4")
