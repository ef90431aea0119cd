"""Writes tests/golden/reference_kat.json: the known-answer vectors of the
reference's own tests, recomputed by restating their PHP expected-value loops
in plain Python (no PHP in this environment).

  conv2d_1x4x4      tests/cuda_conv2d_test.php:19-48
  conv2d_batched    tests/cuda_batched_conv_test.php:18-54
  matmul_2x2        tests/Unit/TensorTest.php:33-39 (literal [19, 22, 43, 50])
  relu              tests/Unit/TensorTest.php:41-46 (literal [0, 0, 2, 0])
  softmax_rows      tests/cuda_attention_test.php:21-38 (includes 100..500 row)
  causal_softmax    tests/cuda_attention_test.php:58-77 (mask -1e9, then softmax)
  scale             tests/cuda_attention_test.php:99-107 (literal)
  softmax_bwd       tests/cuda_attention_test.php:120-138
  attention_full    tests/cuda_attention_full_test.php:18-131 (mt_srand(42) inputs regenerated
                    with an MT19937 restatement of PHP mt_rand; stored in the fixture)

Run:  python tests/golden/make_golden.py
"""
import json
import math
import os


def conv_kat(inp, B, H, W, weight, bias, k=3, stride=1, pad=0):
    oH = (H + 2 * pad - k) // stride + 1
    oW = (W + 2 * pad - k) // stride + 1
    out = []
    for b in range(B):
        for oh in range(oH):
            for ow in range(oW):
                s = bias[0]
                for kh in range(k):
                    for kw in range(k):
                        ih, iw = oh * stride - pad + kh, ow * stride - pad + kw
                        s += inp[b * H * W + ih * W + iw] * weight[kh * k + kw]
                out.append(s)
    return out


def softmax_rows(x, N, M, causal=False):
    out = []
    for i in range(N):
        row = list(x[i * M:(i + 1) * M])
        if causal:
            row = [(-1e9 if j > i else v) for j, v in enumerate(row)]
        mx = max(row)
        e = [math.exp(v - mx) for v in row]
        s = sum(e)
        out += [v / s for v in e]
    return out


class PhpMtRand:
    """MT19937 as PHP 7.1+ uses it for mt_srand()/mt_rand(): init_genrand(seed),
    tempered 32-bit outputs, and mt_rand() = output >> 1 (mt_getrandmax() = 2^31-1).
    Restated from the published Mersenne Twister algorithm."""

    def __init__(self, seed):
        self.mt = [0] * 624
        self.mt[0] = seed & 0xFFFFFFFF
        for i in range(1, 624):
            self.mt[i] = (1812433253 * (self.mt[i - 1] ^ (self.mt[i - 1] >> 30)) + i) & 0xFFFFFFFF
        self.idx = 624

    def _twist(self):
        for i in range(624):
            y = (self.mt[i] & 0x80000000) | (self.mt[(i + 1) % 624] & 0x7FFFFFFF)
            v = self.mt[(i + 397) % 624] ^ (y >> 1)
            if y & 1:
                v ^= 0x9908B0DF
            self.mt[i] = v
        self.idx = 0

    def rand(self):
        if self.idx >= 624:
            self._twist()
        y = self.mt[self.idx]
        self.idx += 1
        y ^= y >> 11
        y ^= (y << 7) & 0x9D2C5680
        y ^= (y << 15) & 0xEFC60000
        y ^= y >> 18
        return (y & 0xFFFFFFFF) >> 1


def php_randn(gen, n):
    """tests/cuda_attention_full_test.php:97-106 (Box-Muller on mt_rand)."""
    out = []
    for _ in range(n):
        u1 = gen.rand() / 2147483647
        u2 = gen.rand() / 2147483647
        out.append(math.sqrt(-2.0 * math.log(u1 or 1e-12)) * math.cos(2.0 * math.pi * u2))
    return out


def attention_kat():
    """tests/cuda_attention_full_test.php:18-26,107-131: Q, K, V from mt_srand(42),
    causal attention N=4, D=8 with the test's own expected-value loop."""
    N, D = 4, 8
    scale = 1.0 / math.sqrt(D)
    g = PhpMtRand(42)
    Q, K, V = php_randn(g, N * D), php_randn(g, N * D), php_randn(g, N * D)
    S = [[sum(Q[i * D + d] * K[j * D + d] for d in range(D)) * scale for j in range(N)] for i in range(N)]
    for i in range(N):
        for j in range(N):
            if j > i:
                S[i][j] = -1e9
    P = []
    for i in range(N):
        mx = max(S[i])
        e = [math.exp(v - mx) for v in S[i]]
        s = sum(e)
        P.append([v / s for v in e])
    O = [sum(P[i][j] * V[j * D + d] for j in range(N)) for i in range(N) for d in range(D)]
    return {"Q": Q, "K": K, "V": V, "N": N, "D": D, "scale": scale, "tol": 1e-4, "expected": O}


def main():
    kernel = [1.0, 0.0, -1.0, 0.0, 1.0, 0.0, -1.0, 0.0, 1.0]
    img = [float(v) for v in range(1, 17)]
    img_rev = [float(v) for v in range(16, 0, -1)]
    sm_in = [1, 2, 3, 4, 5, 2, 2, 2, 2, 2, -1, 0, 1, -1, 0, 100, 200, 300, 400, 500]
    causal_in = [1.0, 2.0, 3.0, 4.0] * 4
    P = [0.2, 0.3, 0.5, 0.1, 0.8, 0.1]
    dP = [1.0, 0.0, 0.0, 0.0, 1.0, 0.0]
    dS = []
    for i in range(2):
        dot = sum(dP[i * 3 + j] * P[i * 3 + j] for j in range(3))
        dS += [P[i * 3 + j] * (dP[i * 3 + j] - dot) for j in range(3)]
    g = {
        "conv2d_1x4x4": {"input": img, "weight": kernel, "bias": [0.0], "C": 1, "H": 4, "W": 4,
                          "outC": 1, "k": 3, "stride": 1, "pad": 0, "tol": 1e-4,
                          "expected": conv_kat(img, 1, 4, 4, kernel, [0.0])},
        "conv2d_batched": {"input": img + img_rev, "weight": kernel, "bias": [0.0], "B": 2, "C": 1, "H": 4,
                            "W": 4, "outC": 1, "k": 3, "stride": 1, "pad": 0, "tol": 1e-4,
                            "expected": conv_kat(img + img_rev, 2, 4, 4, kernel, [0.0])},
        "matmul_2x2": {"a": [1.0, 2.0, 3.0, 4.0], "b": [5.0, 6.0, 7.0, 8.0], "M": 2, "K": 2, "N": 2,
                       "expected": [19.0, 22.0, 43.0, 50.0]},
        "relu": {"x": [-1.0, 0.0, 2.0, -3.0], "expected": [0.0, 0.0, 2.0, 0.0]},
        "softmax_rows": {"x": [float(v) for v in sm_in], "N": 4, "M": 5, "tol": 1e-5,
                         "expected": softmax_rows(sm_in, 4, 5)},
        "causal_softmax": {"x": causal_in, "N": 4, "M": 4, "mask": -1e9, "tol": 1e-5,
                           "expected": softmax_rows(causal_in, 4, 4, causal=True)},
        "scale": {"x": [1.0, 2.0, 3.0, 4.0, 5.0, 6.0], "s": 0.5, "tol": 1e-6,
                  "expected": [0.5, 1.0, 1.5, 2.0, 2.5, 3.0]},
        "softmax_bwd": {"P": P, "dP": dP, "N": 2, "M": 3, "tol": 1e-5, "expected": dS},
        "attention_full": attention_kat(),
    }
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "reference_kat.json")
    with open(path, "w") as f:
        json.dump(g, f, indent=1)
    print(path)


if __name__ == "__main__":
    main()
