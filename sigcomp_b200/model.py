"""Integer entropy-model parameters.

SigComp ships its entropy model as a quantised PyTorch ``state_dict``
(``pretrained_models/{lossless,lossy}.pth``).  The codec never runs the float
model: it runs the integer pipeline that ``load_cpu_decoder``
(sigcomp/cpu_int_inference.py:395-445) derives from that state dict.  This
module derives the same integers:

* embedding ``E_q = clamp(round(E / s_in), -128, 127)`` (cpu_int_inference.py:406-414);
* per linear layer ``W_q`` (int8), ``b_q = round(b / (s_in * s_w))`` (int32) and the
  fixed-point multiplier ``(M0, shift) = frexp(s_in * s_w / s_out)``
  (``_extract_linear`` :350-368, ``float_to_multiplier_shift`` :17-21);
* ReLU on every layer but the last (:429);
* the exponential table ``lut[i] = floor(exp(-i * s_out) * 2**38)`` evaluated in
  50-digit decimal arithmetic (``build_integer_exp_lut``,
  sigcomp/cpu_entropy_coding.py:49-61).

The float-to-integer steps use the same torch operations as the reference so
that rounding of ties and float32 intermediate precision agree bit for bit.
"""

from dataclasses import dataclass, field
from decimal import Decimal, localcontext
import hashlib
import math
import re
import os
from pathlib import Path

import numpy as np

VOCAB = 256
SOS_TOKEN = 256
LUT_BITS = 38
PRECISION = 24

MODEL_DIR = Path(__file__).resolve().parent / "models"


@dataclass
class IntModel:
    """The integer MLP + exp table that defines one SigComp entropy model."""
    embedding: np.ndarray            # int8 [257, emb_dim]
    weights: list                    # int8 [N_l, K_l]
    biases: list                     # int32 [N_l]
    multipliers: np.ndarray          # int64 [L]  (M0, in [0, 2**31])
    shifts: np.ndarray               # int32 [L]  (in [0, 63])
    relu: np.ndarray                 # uint8 [L]
    output_scale: float
    exp_lut: np.ndarray              # int64 [256]
    window_size: int = 64
    name: str = field(default="model")

    @property
    def emb_dim(self):
        return int(self.embedding.shape[1])

    @property
    def num_layers(self):
        return len(self.weights)

    def geometry(self):
        return {
            "window": self.window_size, "emb_dim": self.emb_dim,
            "layers": [tuple(int(x) for x in w.shape) for w in self.weights],
        }

    def digest(self):
        h = hashlib.sha256()
        for arr in [self.embedding, *self.weights, *self.biases, self.multipliers,
                    self.shifts, self.relu, self.exp_lut]:
            h.update(np.ascontiguousarray(arr).tobytes())
        return h.hexdigest()

    def save(self, path):
        arrays = {
            "embedding": self.embedding, "multipliers": self.multipliers,
            "shifts": self.shifts, "relu": self.relu, "exp_lut": self.exp_lut,
            "output_scale": np.float64(self.output_scale),
            "window_size": np.int64(self.window_size),
        }
        for i, (w, b) in enumerate(zip(self.weights, self.biases)):
            arrays[f"w{i}"] = w
            arrays[f"b{i}"] = b
        path = Path(path)
        path.parent.mkdir(parents=True, exist_ok=True)
        tmp = path.with_suffix(".tmp.npz")
        np.savez(tmp, **arrays)
        os.replace(tmp, path)

    @classmethod
    def load_npz(cls, path):
        with np.load(path) as z:
            layers = sum(1 for k in z.files if re.fullmatch(r"w\d+", k))
            return cls(
                embedding=z["embedding"], weights=[z[f"w{i}"] for i in range(layers)],
                biases=[z[f"b{i}"] for i in range(layers)], multipliers=z["multipliers"],
                shifts=z["shifts"], relu=z["relu"], output_scale=float(z["output_scale"]),
                exp_lut=z["exp_lut"], window_size=int(z["window_size"]),
                name=Path(path).stem)


def float_to_multiplier_shift(multiplier):
    """frexp-based fixed-point multiplier (cpu_int_inference.py:17-21)."""
    if multiplier == 0:
        return 0, 0
    significand, exponent = math.frexp(multiplier)
    return int(round(significand * (2 ** 31))), 31 - exponent


def build_exp_lut(output_scale, bits=LUT_BITS):
    """``lut[i] = floor(exp(-i * s) * 2**bits)`` in 50-digit decimal arithmetic
    (cpu_entropy_coding.py:49-61)."""
    scale = float(output_scale)
    if not math.isfinite(scale) or scale < 0:
        raise ValueError("output_scale must be a finite nonnegative number")
    with localcontext() as ctx:
        ctx.prec = 50
        s = Decimal(str(scale))
        mult = Decimal(1 << bits)
        vals = [max(int((Decimal(-i) * s).exp() * mult), 0) for i in range(VOCAB)]
    return np.asarray(vals, dtype=np.int64)


def load_state_dict_model(path, dim=256, num_dec_layers=8, window_size=64):
    """Derive an :class:`IntModel` from a quantised SigComp ``.pth`` state dict."""
    import torch

    dim = 256 if dim is None else int(dim)
    num_dec_layers = 8 if num_dec_layers is None else int(num_dec_layers)
    window_size = 64 if window_size is None else int(window_size)
    if dim < 2 or num_dec_layers < 0 or window_size < 1:
        raise ValueError("Invalid MLP architecture")
    state = torch.load(Path(path), map_location="cpu", weights_only=True)
    try:
        emb = state["decoder.embedding_linear.weight"]
        s_in = float(state["decoder.quant.scale"].item())
        if emb.shape != (257, dim // 2):
            raise ValueError("Checkpoint embedding shape does not match --dim")
        if not math.isfinite(s_in) or s_in <= 0:
            raise ValueError("Invalid embedding quantization scale")
        emb_q = torch.round(emb / s_in).clamp(-128, 127).to(torch.int8).numpy()
        weights, biases, mults, shifts, relu = [], [], [], [], []
        expected_in = (dim // 2) * window_size
        for index in range(num_dec_layers + 1):
            prefix = f"decoder.mlp.{index * 2}"
            weight, bias = state[f"{prefix}._packed_params._packed_params"]
            s_out = float(state[f"{prefix}.scale"].item())
            out_w = dim * 2 if index < num_dec_layers else 256
            if weight.shape != (out_w, expected_in):
                raise ValueError(f"Checkpoint {prefix} shape does not match the geometry")
            if not math.isfinite(s_out) or s_out <= 0:
                raise ValueError(f"Invalid quantization scale for {prefix}")
            if weight.dtype != torch.qint8 or weight.qscheme() not in (
                    torch.per_tensor_affine, torch.per_tensor_symmetric):
                raise ValueError("Expected per-tensor quantized int8 linear weights")
            w_q = weight.int_repr()
            bias_scale = s_in * weight.q_scale()
            if bias is None:
                b_q = torch.zeros(w_q.shape[0], dtype=torch.int32)
            else:
                b_q = torch.round(bias.detach().cpu() / bias_scale).to(torch.int32)
            m0, sh = float_to_multiplier_shift(bias_scale / s_out)
            if not 0 <= m0 <= (1 << 31) or not 0 <= sh <= 63:
                raise ValueError("quantized multiplier out of range")
            weights.append(np.ascontiguousarray(w_q.numpy()))
            biases.append(np.ascontiguousarray(b_q.numpy()))
            mults.append(m0)
            shifts.append(sh)
            relu.append(1 if index < num_dec_layers else 0)
            s_in = s_out
            expected_in = out_w
        layers = sum(k.startswith("decoder.mlp.") and k.endswith("._packed_params._packed_params")
                     for k in state)
        if layers != num_dec_layers + 1:
            raise ValueError("Checkpoint layer count does not match --num-dec-layers")
    except KeyError as exc:
        raise ValueError(f"Incomplete or incompatible quantized MLP checkpoint: {exc}") from exc
    return IntModel(
        embedding=np.ascontiguousarray(emb_q), weights=weights, biases=biases,
        multipliers=np.asarray(mults, dtype=np.int64), shifts=np.asarray(shifts, dtype=np.int32),
        relu=np.asarray(relu, dtype=np.uint8), output_scale=s_in,
        exp_lut=build_exp_lut(s_in), window_size=window_size, name=Path(path).stem)


def load_model(path=None, name="lossless", dim=None, num_dec_layers=None, window_size=None):
    """Load a model from a ``.pth`` state dict or an exported ``.npz``.

    With no path, the exported copy of the bundled model ``name`` is used
    (written by ``__graft_entry__.build()`` from the reference's bundled
    ``.pth``).
    """
    if path is None:
        path = MODEL_DIR / f"{name}.npz"
        if not path.exists():
            raise FileNotFoundError(
                f"exported model {path} is missing; run __graft_entry__.build() where the "
                "SigComp .pth files are available, or pass model_path")
    path = Path(path)
    if path.suffix == ".npz":
        return IntModel.load_npz(path)
    return load_state_dict_model(path, dim=dim, num_dec_layers=num_dec_layers,
                                 window_size=window_size)


def random_model(seed=0, emb_dim=128, window=64, hidden=512, num_dec_layers=8, vocab_out=256,
                 weight_scale=1.0):
    """A seeded random integer model with the bundled geometry, for kernel tests.

    Multipliers and shifts are chosen so activations stay spread over the int8
    range (neither saturated nor all zero), which exercises the requantisation
    edge cases.
    """
    rng = np.random.default_rng(seed)
    emb = rng.integers(-128, 128, size=(257, emb_dim), dtype=np.int64).astype(np.int8)
    weights, biases, mults, shifts, relu = [], [], [], [], []
    k = emb_dim * window
    for i in range(num_dec_layers + 1):
        n = hidden if i < num_dec_layers else vocab_out
        w = np.clip(np.rint(rng.normal(0, 40 * weight_scale, size=(n, k))), -128, 127).astype(np.int8)
        b = rng.integers(-5000, 5000, size=n).astype(np.int32)
        # typical |acc| ~ 40 * 70 * sqrt(k); aim the output spread at ~ +-100
        target = 100.0 / (40 * 70 * math.sqrt(k))
        m0, sh = float_to_multiplier_shift(target * float(rng.uniform(0.7, 1.4)))
        weights.append(w)
        biases.append(b)
        mults.append(m0)
        shifts.append(sh)
        relu.append(1 if i < num_dec_layers else 0)
        k = n
    scale = 0.05
    return IntModel(
        embedding=emb, weights=weights, biases=biases,
        multipliers=np.asarray(mults, dtype=np.int64), shifts=np.asarray(shifts, dtype=np.int32),
        relu=np.asarray(relu, dtype=np.uint8), output_scale=scale,
        exp_lut=build_exp_lut(scale), window_size=window, name=f"random{seed}")
