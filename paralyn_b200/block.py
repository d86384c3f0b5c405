"""The pre-LN transformer encoder block of the reference's examples, on the tensor provider.

Reference: examples/native/transformer_block.{cpp,py} and docs/transformer-operators.md:
195-258. x [T, d] -> LayerNorm -> fused QKV projection [T, 3d] + bias -> per-head scores
Q_h K_h^T (strided head views of the QKV output, no copies) -> causal softmax with scale
fl32(1/sqrt(d_head)) -> P_h V_h written through strides into the concatenated [T, d]
attention output -> output projection + bias -> residual add -> LayerNorm -> MLP up
projection + bias + tanh-GELU -> down projection + bias -> residual add.

`run()` enqueues the reference's 15 launches; `run(fused=True)` runs the same block in
11, with every bias (and the GELU) in the epilogue of its GEMM
(pr_b200_matmul_bias_activation_f32), bit-identical to the 15-launch form. After
`prepare_weights()` the four projections read their weights' prepared forms
(pr_b200_matmul_prepare_f32, made once), so no block splits a weight again; the results
stay bit-identical.
Weights come from the seeded device stream (scales 0.125 / 0.0625, gamma 1 +- 0.25,
biases +- 0.25, as the reference example uses); all buffers stay on the device.
"""
import math

import numpy as np

from . import b200
from .tensor import (Activation, TensorDescriptor, add_into, batched_matmul_into, bias_activation_into,
                     layer_norm_into, matmul_into, operators_of, softmax_rows_into)


class EncoderBlock:
    WEIGHTS = ("gamma1", "beta1", "w_qkv", "b_qkv", "w_o", "b_o", "gamma2", "beta2", "w_1", "b_1", "w_2", "b_2")

    def __init__(self, context, tokens, d_model, heads, d_ff, *, causal=True, seed=2026, epsilon=1e-5):
        if d_model % heads:
            raise ValueError("d_model must be a multiple of heads")
        self.context, self.causal, self.epsilon = context, causal, epsilon
        self.T, self.D, self.H, self.F = tokens, d_model, heads, d_ff
        self.DH = d_model // heads
        self.scale = float(np.float32(1.0 / math.sqrt(self.DH)))
        self.ops = operators_of(context)
        T, D, H, F = tokens, d_model, heads, d_ff
        self.shapes = {
            "x": (T, D), "gamma1": (D,), "beta1": (D,), "w_qkv": (D, 3 * D), "b_qkv": (3 * D,),
            "w_o": (D, D), "b_o": (D,), "gamma2": (D,), "beta2": (D,), "w_1": (D, F), "b_1": (F,),
            "w_2": (F, D), "b_2": (D,),
            "ln1": (T, D), "qkv": (T, 3 * D), "qkv_b": (T, 3 * D), "scores": (H, T, T), "probs": (H, T, T),
            "attn": (T, D), "proj": (T, D), "proj_b": (T, D), "h1": (T, D), "ln2": (T, D), "ff1": (T, F),
            "ff1_g": (T, F), "ff2": (T, D), "ff2_b": (T, D), "out": (T, D)}
        self.buf = {name: context.buffer(4 * int(np.prod(shape))) for name, shape in self.shapes.items()}
        self._descriptors = {}
        self.prepared = {}  # weight name -> b200.PreparedMatrix
        fills = {"x": (1.0, 0.0), "w_qkv": (0.125, 0.0), "w_o": (0.125, 0.0), "w_1": (0.125, 0.0),
                 "w_2": (0.0625, 0.0), "b_qkv": (0.25, 0.0), "b_o": (0.25, 0.0), "b_1": (0.25, 0.0),
                 "b_2": (0.25, 0.0), "beta1": (0.25, 0.0), "beta2": (0.25, 0.0)}
        events = []
        for i, (name, (p0, _)) in enumerate(fills.items()):
            events.append(b200.fill_synthetic_into(self.ops.queue, self.d(name), seed=seed + i, p0=p0))
        for e in events:
            if e is not None:
                e.wait()
                e.close()
        for name in ("gamma1", "gamma2"):  # 1 +- 0.25
            g = 1.0 + 0.25 * (np.arange(D, dtype=np.float32) % 7 - 3) / 3
            self.buf[name].write(g.astype(np.float32))

    def d(self, name, shape=None, offset=0, strides=None):
        key = (name, shape, offset, strides)
        desc = self._descriptors.get(key)
        if desc is None:  # built once: repeated blocks reuse the descriptors and their records
            desc = self._descriptors[key] = TensorDescriptor(self.buf[name], shape or self.shapes[name], offset,
                                                             strides)
        return desc

    def prepare_weights(self):
        """Prepare the projection weights once; later runs skip their split passes.
        A weight written after this is not seen by the projections (prepare again)."""
        self.release_prepared()
        for name in ("w_qkv", "w_o", "w_1", "w_2"):
            k, n = self.shapes[name]
            self.prepared[name] = b200.PreparedMatrix(self.ops.queue, self.ops.module, self.context, self.d(name),
                                                      k=k, n=n)

    def release_prepared(self):
        while self.prepared:
            self.prepared.popitem()[1].close()

    def flops(self):
        """GEMM flops of one block (projections, scores, P V, MLP)."""
        T, D, H, F, DH = self.T, self.D, self.H, self.F, self.DH
        return 2 * T * D * 3 * D + 2 * 2 * H * T * T * DH + 2 * T * D * D + 2 * 2 * T * D * F

    def run(self, fused=False):
        """Enqueue one block; returns its events (15, or 11 when fused) in launch order."""
        q, m, d = self.ops.queue, self.ops.module, self.d
        T, D, H, F, DH = self.T, self.D, self.H, self.F, self.DH

        def dense(a, w, bias, out, pre, n, k, activation=Activation.NONE):
            prepared = self.prepared.get(w)
            if fused and prepared:
                return [b200.matmul_prepared_bias_activation_into(q, m, d(a), prepared.descriptor, d(out), d(bias),
                                                                  m=T, n=n, k=k, activation=activation)]
            if fused:
                return [b200.matmul_bias_activation_into(q, m, d(a), d(w), d(out), d(bias), m=T, n=n, k=k,
                                                         activation=activation)]
            product = (b200.matmul_prepared_into(q, m, d(a), prepared.descriptor, d(pre), m=T, n=n, k=k)
                       if prepared else matmul_into(q, m, d(a), d(w), d(pre), m=T, n=n, k=k))
            return [product, bias_activation_into(q, m, d(pre), d(bias), d(out), activation=activation)]

        events = [layer_norm_into(q, m, d("x"), d("gamma1"), d("beta1"), d("ln1"), epsilon=self.epsilon)]
        events += dense("ln1", "w_qkv", "b_qkv", "qkv_b", "qkv", 3 * D, D)
        # Q_h [H,T,DH] strides [DH, 3D, 1]; K_h^T [H,DH,T] strides [DH, 1, 3D] at column D
        events.append(batched_matmul_into(q, m, d("qkv_b", (H, T, DH), 0, (DH, 3 * D, 1)),
                                          d("qkv_b", (H, DH, T), 4 * D, (DH, 1, 3 * D)), d("scores"),
                                          batch=H, m=T, n=T, k=DH))
        events.append(softmax_rows_into(q, m, d("scores"), d("probs"), scale=self.scale, causal=self.causal))
        # P_h V_h with V_h at column 2D, into the concatenated [T, D] output (strides [DH, D, 1])
        events.append(batched_matmul_into(q, m, d("probs"), d("qkv_b", (H, T, DH), 8 * D, (DH, 3 * D, 1)),
                                          d("attn", (H, T, DH), 0, (DH, D, 1)), batch=H, m=T, n=DH, k=T))
        events += dense("attn", "w_o", "b_o", "proj_b", "proj", D, D)
        events.append(add_into(q, m, d("x"), d("proj_b"), d("h1")))
        events.append(layer_norm_into(q, m, d("h1"), d("gamma2"), d("beta2"), d("ln2"), epsilon=self.epsilon))
        events += dense("ln2", "w_1", "b_1", "ff1_g", "ff1", F, D, Activation.GELU_TANH)
        events += dense("ff1_g", "w_2", "b_2", "ff2_b", "ff2", D, F)
        events.append(add_into(q, m, d("h1"), d("ff2_b"), d("out")))
        return [e for e in events if e is not None]

    def read(self, name):
        return np.frombuffer(self.buf[name].read(), np.float32).reshape(self.shapes[name]).copy()

    def close(self):
        self.release_prepared()
        for b in self.buf.values():
            b.close()
