"""CPU restatement of the reference SigLIP vision encoder -- TEST INFRASTRUCTURE ONLY.

numpy (fp32) restatement of siglip_forward (common/vision/siglip.c:71-156 of
tmzt/smol-genius): patch embedding (smol_conv2d with kernel = stride = patch,
conv2d.c:13-95: im2col rows ordered (channel, ky, kx)), learnable position embeddings,
then per layer LayerNorm -> Q/K/V (with bias) -> bidirectional attention over all
patches -> output projection -> residual, LayerNorm -> fc1 -> GELU (tanh form,
activation.c:29-36) -> fc2 -> residual; post-LayerNorm (layernorm.c:17-124).  The
attention goes through the C restatement (pyoracle: smol_oracle.c).

`device_formats=True` rounds every intermediate the device keeps in 16 bits the same
way (LayerNorm outputs, the attention output and the GELU output bf16; Q, K bf16; V
fp16; patch pixels bf16), so that the device path is compared on identical operands;
`False` is the reference's all-fp32 arithmetic.  Matrices are bf16-valued (stored as
the rounded fp32 values), biases and norm weights fp32.

Pinned to the reference's siglip_forward itself (SIGLIP_PIN_CASES below, run by the
compiled reference on the same weights): tests/test_siglip_oracle.py, live and against
tests/golden/siglip_cases.npz; the windowed encoder-layer composition in
tests/test_encoder_layers_oracle.py.

Only tests/ import this module.
"""
from __future__ import annotations

import struct

import numpy as np

import pyoracle


def layer_norm(x: np.ndarray, w: np.ndarray, b: np.ndarray, eps: float) -> np.ndarray:
    """smol_layer_norm (layernorm.c:17-124): (x - mean) * 1/sqrtf(var + eps) * w + b per row,
    var the mean of squared deviations."""
    x = x.astype(np.float32)
    n = np.float32(x.shape[-1])
    mean = (np.sum(x, axis=-1, keepdims=True, dtype=np.float32) / n).astype(np.float32)
    d = (x - mean).astype(np.float32)
    var = (np.sum(d * d, axis=-1, keepdims=True, dtype=np.float32) / n).astype(np.float32)
    inv = (np.float32(1.0) / np.sqrt(var + np.float32(eps))).astype(np.float32)
    return ((d * inv) * w + b).astype(np.float32)


def gelu_tanh(x: np.ndarray) -> np.ndarray:
    """smol_gelu (activation.c:29-36): 0.5*x*(1 + tanh(0.7978845608028654*(x + 0.044715*x^3)))."""
    x3 = (x * x * x).astype(np.float32)
    inner = (np.float32(0.7978845608028654) * (x + np.float32(0.044715) * x3)).astype(np.float32)
    return (np.float32(0.5) * x * (np.float32(1.0) + np.tanh(inner, dtype=np.float32))).astype(np.float32)


def f16(x: np.ndarray) -> np.ndarray:
    return x.astype(np.float16).astype(np.float32)


def unfold_patches(image: np.ndarray, patch: int) -> np.ndarray:
    """[3, H, W] -> [n_patches, 3*patch*patch]: im2col's rows (conv2d.c:13-50) as columns,
    patches in row-major grid order (the reshape of siglip.c:45-56)."""
    c, h, w = image.shape
    ph, pw = h // patch, w // patch
    t = image[:, :ph * patch, :pw * patch].reshape(c, ph, patch, pw, patch)
    return t.transpose(1, 3, 0, 2, 4).reshape(ph * pw, c * patch * patch).astype(np.float32)


class SiglipOracle:
    """A seeded SigLIP encoder and its forward pass."""

    def __init__(self, hidden=128, heads=2, ffn=256, layers=2, patch=16, image=64, eps=1e-6, seed=0):
        rng = np.random.default_rng(seed)
        self.H, self.NH, self.F, self.L, self.P, self.eps = hidden, heads, ffn, layers, patch, eps
        self.HD = hidden // heads
        self.image = image
        self.n_pos = (image // patch) ** 2
        kin = 3 * patch * patch

        def mat(rows, cols, sc):
            return pyoracle.round_bf16((rng.standard_normal((rows, cols)) * sc).astype(np.float32))

        def vec(n, mean, sd):
            return (mean + sd * rng.standard_normal(n)).astype(np.float32)

        self.patch_w = mat(hidden, kin, 1 / np.sqrt(kin))          # [hidden, 3, p, p] flattened
        self.patch_b = vec(hidden, 0.0, 0.02)
        self.pos = vec(self.n_pos * hidden, 0.0, 0.5).reshape(self.n_pos, hidden)
        self.layers = []
        for _ in range(layers):
            self.layers.append({
                "ln1_w": vec(hidden, 1.0, 0.05), "ln1_b": vec(hidden, 0.0, 0.02),
                "wq": mat(hidden, hidden, 1 / np.sqrt(hidden)), "bq": vec(hidden, 0.0, 0.02),
                "wk": mat(hidden, hidden, 1 / np.sqrt(hidden)), "bk": vec(hidden, 0.0, 0.02),
                "wv": mat(hidden, hidden, 1 / np.sqrt(hidden)), "bv": vec(hidden, 0.0, 0.02),
                "wo": mat(hidden, hidden, 1 / np.sqrt(hidden)), "bo": vec(hidden, 0.0, 0.02),
                "ln2_w": vec(hidden, 1.0, 0.05), "ln2_b": vec(hidden, 0.0, 0.02),
                "fc1": mat(ffn, hidden, 1 / np.sqrt(hidden)), "b1": vec(ffn, 0.0, 0.02),
                "fc2": mat(hidden, ffn, 1 / np.sqrt(ffn)), "b2": vec(hidden, 0.0, 0.02),
            })
        self.post_w = vec(hidden, 1.0, 0.05)
        self.post_b = vec(hidden, 0.0, 0.02)
        self.o = pyoracle.oracle()

    def embed(self, images: np.ndarray, device_formats: bool) -> np.ndarray:
        """Patch embedding + position embeddings (siglip.c:24-100): [n_img, n_pos, hidden]."""
        out = []
        for img in images:
            u = unfold_patches(img, self.P)
            if device_formats:
                u = pyoracle.round_bf16(u)
            out.append((u @ self.patch_w.T + self.patch_b + self.pos).astype(np.float32))
        return np.stack(out)

    def layer(self, x: np.ndarray, l: int, device_formats: bool, window_starts=None) -> np.ndarray:
        """One encoder layer over [n_img, seq, hidden] (siglip.c:112-147); window_starts
        limits the attention to windows, as the Qwen3-ASR audio encoder's layers do
        (encoder.c:449-484)."""
        lw = self.layers[l]
        r16 = pyoracle.round_bf16 if device_formats else (lambda a: a)
        v16 = f16 if device_formats else (lambda a: a)
        n_img, seq, H = x.shape
        out = np.empty_like(x)
        scale = np.float32(1.0 / np.sqrt(np.float32(self.HD)))
        for i in range(n_img):
            xi = x[i]
            xn = r16(layer_norm(xi, lw["ln1_w"], lw["ln1_b"], self.eps))
            q = r16((xn @ lw["wq"].T + lw["bq"]).astype(np.float32))
            k = r16((xn @ lw["wk"].T + lw["bk"]).astype(np.float32))
            v = v16((xn @ lw["wv"].T + lw["bv"]).astype(np.float32))
            a = self.o.bidirectional_attention(q, k, v, seq, self.NH, self.HD, scale,
                                               [0, seq] if window_starts is None else window_starts)
            a = r16(a)
            xi = (xi + (a @ lw["wo"].T + lw["bo"])).astype(np.float32)
            xn = r16(layer_norm(xi, lw["ln2_w"], lw["ln2_b"], self.eps))
            h = r16(gelu_tanh((xn @ lw["fc1"].T + lw["b1"]).astype(np.float32)))
            out[i] = (xi + (h @ lw["fc2"].T + lw["b2"])).astype(np.float32)
        return out

    def encoder_layers(self, x: np.ndarray, device_formats: bool = True, window_starts=None) -> np.ndarray:
        """The layer stack alone over [batch, seq, hidden] (no patch embedding, no post-LN)."""
        for l in range(self.L):
            x = self.layer(x, l, device_formats, window_starts)
        return x

    def forward(self, images: np.ndarray, device_formats: bool = True) -> np.ndarray:
        """siglip_forward for a batch of [3, image, image] images: [n_img, n_pos, hidden]."""
        x = self.embed(images, device_formats)
        for l in range(self.L):
            x = self.layer(x, l, device_formats)
        return layer_norm(x, self.post_w, self.post_b, self.eps)

    def images(self, n: int, seed: int) -> np.ndarray:
        """Seeded pixel values in [-1, 1] (the range of the exports' normalised images)."""
        rng = np.random.default_rng(seed)
        return rng.uniform(-1.0, 1.0, (n, 3, self.image, self.image)).astype(np.float32)

    def write_weights_file(self, path, images: np.ndarray) -> None:
        """Input of tests/dropin/siglip_weights_main.c (its header comment gives the format)."""
        f32 = lambda a: np.ascontiguousarray(a, dtype=np.float32).tobytes()   # noqa: E731
        with open(path, "wb") as f:
            f.write(b"SGLP")
            f.write(struct.pack("<8i", self.H, self.NH, self.F, self.L, self.P, self.image, self.n_pos, len(images)))
            f.write(struct.pack("<f", self.eps))
            f.write(f32(self.patch_w))
            f.write(f32(self.patch_b))
            f.write(f32(self.pos))
            for lw in self.layers:
                for name in ("ln1_w", "ln1_b", "wq", "bq", "wk", "bk", "wv", "bv", "wo", "bo", "ln2_w", "ln2_b",
                             "fc1", "b1", "fc2", "b2"):
                    f.write(f32(lw[name]))
            f.write(f32(self.post_w))
            f.write(f32(self.post_b))
            f.write(f32(images))


# Cases that pin this restatement to the reference encoder (oracle/_ref/siglip_weights_ref).
SIGLIP_PIN_CASES = {
    "h128-p16": {"hidden": 128, "heads": 2, "ffn": 256, "layers": 2, "patch": 16, "image": 64, "seed": 1},
    "h192-p8": {"hidden": 192, "heads": 3, "ffn": 512, "layers": 3, "patch": 8, "image": 64, "seed": 2},
}


def siglip_pin_case(name: str):
    """(encoder, images) of a pin case: two seeded images."""
    m = SiglipOracle(**SIGLIP_PIN_CASES[name])
    return m, m.images(2, 5)
