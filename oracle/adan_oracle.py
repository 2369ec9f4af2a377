"""CPU restatement of the reference's Adan (test infrastructure only: the checker of
libcvhrf's cvhrf_adan, never part of the product path).

Follows utils/optimizer.py:
  * step bookkeeping and bias corrections :415-423 (group['step'] += 1, 1 - beta^step);
  * neg_pre_grad initialisation :436-438 (-clip * grad on a group's first step);
  * the global-norm clip :387-407 (sqrt of the sum of all grad^2; clamp(max / (norm +
    eps of the last group), max=1));
  * the per-tensor update of _single_tensor_adan :487-542 (the foreach path :545-611
    performs the same operations in the same order).
float32 numpy arithmetic, one operation at a time.  Pinned to tests/golden/adan_*.npz,
which were produced by the reference's own Adan (tests/golden/make_adan_golden.py).
"""
import math

import numpy as np

f32 = np.float32


class AdanOracle:
    def __init__(self, params, lrs, betas=(0.98, 0.92, 0.99), eps=1e-8, weight_decay=0.0, max_grad_norm=0.0,
                 no_prox=False):
        self.p = [np.array(x, dtype=f32) for x in params]
        self.lrs = [float(l) for l in lrs]
        self.betas = tuple(float(b) for b in betas)
        # torch receives Python doubles and rounds each scalar to float once: beta (mul_),
        # 1 - beta (alpha / value), step sizes, 1 -/+ lr wd are formed in double first
        self.b1, self.b2, self.b3 = (f32(b) for b in self.betas)
        self.omb1, self.omb2, self.omb3 = (f32(1.0 - b) for b in self.betas)
        self.eps, self.wd, self.mgn, self.no_prox = float(eps), float(weight_decay), max_grad_norm, no_prox
        self.m = [np.zeros_like(x) for x in self.p]
        self.v = [np.zeros_like(x) for x in self.p]
        self.diff = [np.zeros_like(x) for x in self.p]
        self.npg = [None for _ in self.p]
        self.t = 0

    def step(self, grads):
        grads = [np.array(g, dtype=f32) for g in grads]
        clip = f32(1.0)
        if self.mgn > 0:
            total = f32(0.0)
            for g in grads:
                total = f32(total + np.sum(g * g, dtype=f32))
            norm = f32(math.sqrt(total))
            clip = f32(min(f32(self.mgn) / f32(norm + f32(self.eps)), f32(1.0)))
        self.t += 1
        b1, b2, b3 = self.betas
        bc1 = 1.0 - b1 ** self.t
        bc2 = 1.0 - b2 ** self.t
        bc3s = f32(math.sqrt(1.0 - b3 ** self.t))
        for k, g0 in enumerate(grads):
            if self.npg[k] is None or self.t == 1:
                self.npg[k] = (g0 * -clip).astype(f32)
            g = (g0 * clip).astype(f32)
            d = (self.npg[k] + g).astype(f32)
            self.m[k] = (self.m[k] * self.b1 + self.omb1 * g).astype(f32)
            self.diff[k] = (self.diff[k] * self.b2 + self.omb2 * d).astype(f32)
            d = (d * self.b2 + g).astype(f32)
            self.v[k] = (self.v[k] * self.b3 + self.omb3 * d * d).astype(f32)
            denom = (np.sqrt(self.v[k]) / bc3s + f32(self.eps)).astype(f32)
            lr = self.lrs[k]
            step_size_diff = f32(lr * b2 / bc2)
            step_size = f32(lr / bc1)
            p = self.p[k]
            if self.no_prox:
                p = (p * f32(1 - lr * self.wd)).astype(f32)
                p = (p + (-step_size) * self.m[k] / denom).astype(f32)
                p = (p + (-step_size_diff) * self.diff[k] / denom).astype(f32)
            else:
                p = (p + (-step_size) * self.m[k] / denom).astype(f32)
                p = (p + (-step_size_diff) * self.diff[k] / denom).astype(f32)
                p = (p / f32(1 + lr * self.wd)).astype(f32)
            self.p[k] = p
            self.npg[k] = (-g).astype(f32)
