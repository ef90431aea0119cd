"""The training workloads the library is measured and checked on.

Each workload is a ZillaPHP Sequential (src/NN/Sequential.php) written as
layer rows {kind, a, b, c} of the fused-step ABI (include/zilla_b200.h):
1 Conv2D 3x3 stride 1 (in, out, padding), 2 ReLU, 3 MaxPool2D 2x2/2,
4 Linear (in, out).  Flatten is implicit (NCHW order, src/Tensor/Tensor.php:958-981).
"""
from __future__ import annotations

from dataclasses import dataclass, field

CONV, RELU, POOL, LINEAR = 1, 2, 3, 4
SGD, ADAM = 1, 2


@dataclass(frozen=True)
class Workload:
    name: str
    layers: tuple
    batch: int                 # global batch
    in_shape: tuple            # (C, H, W)
    classes: int
    optimizer: int             # SGD or ADAM
    lr: float
    precision: int = 0         # 0 fp32 CUDA cores, 1 bf16 tensor cores (fp32 master)
    input_dist: str = "uniform01"
    notes: str = ""
    adam: tuple = field(default=(0.9, 0.999, 1e-8))

    @property
    def in_features(self) -> int:
        c, h, w = self.in_shape
        return c * h * w

    def spec(self) -> list[list[int]]:
        return [list(r) for r in self.layers]


MLP = Workload(
    "mlp_784_128_10", ((LINEAR, 784, 128, 0), (RELU, 0, 0, 0), (LINEAR, 128, 10, 0)),
    batch=64, in_shape=(1, 28, 28), classes=10, optimizer=SGD, lr=0.1,
    notes="MLP 784->128->ReLU->10, fp32, batch 64, SGD 0.1")

CNN_SMALL = Workload(
    "cnn_1x8_pool_fc", ((CONV, 1, 8, 0), (RELU, 0, 0, 0), (POOL, 0, 0, 0), (LINEAR, 8 * 13 * 13, 10, 0)),
    batch=64, in_shape=(1, 28, 28), classes=10, optimizer=SGD, lr=0.05,
    notes="Conv(1->8,3x3,p0)+ReLU -> MaxPool 2x2 -> Linear(1352->10), fp32, batch 64, SGD 0.05")

CNN_LARGE = Workload(
    "large_cnn", ((CONV, 1, 32, 1), (RELU, 0, 0, 0), (CONV, 32, 64, 1), (RELU, 0, 0, 0), (POOL, 0, 0, 0),
                  (CONV, 64, 128, 1), (RELU, 0, 0, 0), (POOL, 0, 0, 0),
                  (LINEAR, 128 * 7 * 7, 256, 0), (RELU, 0, 0, 0), (LINEAR, 256, 10, 0)),
    batch=8192, in_shape=(1, 28, 28), classes=10, optimizer=ADAM, lr=1e-3, precision=1,
    notes="Conv(1->32)+ReLU -> Conv(32->64)+ReLU -> Pool -> Conv(64->128)+ReLU -> Pool -> "
          "Linear(6272->256)+ReLU -> Linear(256->10); fp32 master weights, bf16 tensor-core conv/GEMM; "
          "global batch 8192; Adam 1e-3")

AUDIO_CNN = Workload(
    "audio_kws_cnn", ((CONV, 1, 16, 1), (RELU, 0, 0, 0), (POOL, 0, 0, 0), (CONV, 16, 32, 1), (RELU, 0, 0, 0),
                      (POOL, 0, 0, 0), (CONV, 32, 64, 1), (RELU, 0, 0, 0), (POOL, 0, 0, 0),
                      (LINEAR, 64 * 8 * 12, 12, 0)),
    batch=4096, in_shape=(1, 64, 101), classes=12, optimizer=ADAM, lr=1e-3, input_dist="normal_m4_s2",
    notes="log-mel 1x64x101 ~ N(-4, 2^2); 3x[Conv+ReLU+Pool] -> Linear(6144->12); fp32; global batch 4096; Adam 1e-3")

WORKLOADS = {w.name: w for w in (MLP, CNN_SMALL, CNN_LARGE, AUDIO_CNN)}


@dataclass(frozen=True)
class LmWorkload:
    """A decoder-only Transformer LM (src/Transformers/TransformerLM.php)."""
    name: str
    vocab: int
    dim: int
    heads: int
    layers: int
    max_seq: int
    ffn: int
    batch: int                 # sequences per step
    seq: int                   # tokens per sequence
    lr: float
    optimizer: int = ADAM
    adam: tuple = field(default=(0.9, 0.999, 1e-8))
    notes: str = ""

    @property
    def rows(self) -> int:
        return self.batch * self.seq


TRANSFORMER_LM = LmWorkload(
    "char_transformer_lm", vocab=65, dim=128, heads=4, layers=2, max_seq=128, ffn=512, batch=64, seq=128, lr=3e-4,
    notes="vocab 65, d 128, 4 heads (head dim 32), 2 pre-LN blocks, FFN 512 ReLU, learned positions, "
          "seq 128, batch 64, causal attention, cross-entropy, Adam 3e-4; fp32")


def lm_param_count(w: LmWorkload) -> int:
    D, F = w.dim, w.ffn
    per_block = 4 * (D * D + D) + D * F + F + F * D + D + 4 * D
    return w.vocab * D + w.max_seq * D + 2 * D + D * w.vocab + w.vocab + w.layers * per_block


def lm_flops_per_token(w: LmWorkload) -> float:
    """Algorithmic FLOPs of one training step per token: 3x the forward's
    2*M*N*K for every projection, FFN and head GEMM, plus the causal
    attention contractions (q k^T and P v over the T(T+1)/2 kept scores,
    three contractions' worth each in the backward)."""
    D, F, V, T = w.dim, w.ffn, w.vocab, w.seq
    dense = w.layers * (4 * D * D + 2 * D * F) + D * V
    attn = w.layers * 2 * D * (T + 1) / 2        # per token: QK^T and PV over ~T/2 keys
    return 2 * 3 * dense + 2 * 3 * attn


def param_count(w: Workload) -> int:
    n = 0
    c, h, wd = w.in_shape
    for kind, a, b, p in w.layers:
        if kind == CONV:
            n += b * a * 9 + b
            c, h, wd = b, h + 2 * p - 2, wd + 2 * p - 2
        elif kind == POOL:
            h, wd = (h - 2) // 2 + 1, (wd - 2) // 2 + 1
        elif kind == LINEAR:
            n += a * b + b
            c, h, wd = b, 1, 1
    return n


def flops_per_sample(w: Workload) -> float:
    """Algorithmic FLOPs of one training step per sample: 2*M*N*K for each
    forward, input-gradient and weight-gradient contraction; the first
    layer's input gradient is not computed."""
    total = 0.0
    c, h, wd = w.in_shape
    first = True
    for kind, a, b, p in w.layers:
        if kind == CONV:
            oh, ow = h + 2 * p - 2, wd + 2 * p - 2
            mac = oh * ow * b * a * 9
            total += 2 * mac * (2 if first else 3)
            c, h, wd = b, oh, ow
            first = False
        elif kind == POOL:
            h, wd = (h - 2) // 2 + 1, (wd - 2) // 2 + 1
        elif kind == LINEAR:
            total += 2 * a * b * (2 if first else 3)
            c, h, wd = b, 1, 1
            first = False
    return total
