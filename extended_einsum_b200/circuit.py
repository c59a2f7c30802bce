"""Folded quad-tree probabilistic circuit executed on the B200 kernels.

This is the circuit that the reference's cirkit demo builds (categorical
inputs, alternating Hadamard products and CP sum layers, demo/cirkit.py:131-187)
in the form FoldSameShapedOperations gives it (preprocess.py:1310-1393): one
folded sum layer per tree level, 'dac,dbc->dab' over (F, B, K) x (F, K, K),
with the folded Hadamard product of the two halves of the previous level in
between (slices + 'cab,cab->cab', see the folded program of a quad-tree
circuit), and a root sum 'ab,cb->ac'.

Per forward pass the launches are:
  1  log-softmax of the categorical logits over the states      (xe_softmax, log output)
  L  softmax of each level's sum-layer logits                     (xe_softmax)
  1  first CP sum layer over every state of each variable: the
     state table T[f, s, :] (F0 x states rows instead of F0 x B)  (xe_logspace_gemm)
  1  second CP sum layer, its A rows the Hadamard product of two
     gathered state-table rows                                    (xe_logspace_gemm_gather_pair)
  L-2 CP sum layers, the Hadamard product fused into the A operand (xe_logspace_gemm, a2)
  1  root softmax + 1 root sum layer                              (xe_softmax, xe_logspace_gemm)
and the whole sequence can be captured in one CUDA graph.

A row of the first layer depends on the sample only through the pixel value of
its variable, so its output for sample b is row pixels[b, var[f]] of the state
table, computed by the same kernel on the same row: the values are those of the
per-sample layer.  For batches smaller than half the states the first layer
runs per sample instead, with the categorical gather fused into it
(xe_logspace_gemm_gather).  Every step is differentiable: the backward of a
fused gather scatters its row gradients back into the table.

Layout in HBM (fp32, contiguous): level output (F, B, K) with the batch
inner to the fold, so that the two Hadamard halves of level l+1 are the two
contiguous halves [0, F/2) and [F/2, F) of level l's output.
"""

from __future__ import annotations

import importlib
import math
from dataclasses import dataclass

import torch

from . import ops


def quad_tree_leaf_order(height: int, width: int) -> list[int]:
    """Pixel variable of each leaf fold.

    The region of fold f at level l+1 is the union of folds f and f + F_{l+1}
    of level l, so the bits of a leaf index, from the lowest, choose the
    half at each split from the root down.  Splits alternate between rows
    and columns (the quad-tree region graph), each halving the region.
    """
    variables = height * width
    if variables & (variables - 1) or height & (height - 1) or width & (width - 1):
        raise ValueError("the quad-tree circuit needs power-of-two height and width")
    levels = int(math.log2(variables))
    order = []
    for leaf in range(variables):
        r0, r1, c0, c1 = 0, height, 0, width
        split_rows = height >= width
        for bit in range(levels):
            choose_second = (leaf >> bit) & 1
            if split_rows and r1 - r0 > 1 or c1 - c0 == 1:
                mid = (r0 + r1) // 2
                r0, r1 = (mid, r1) if choose_second else (r0, mid)
            else:
                mid = (c0 + c1) // 2
                c0, c1 = (mid, c1) if choose_second else (c0, mid)
            split_rows = not split_rows
        order.append(r0 * width + c0)
    return order


@dataclass(frozen=True)
class QuadTreeCircuit:
    height: int = 32
    width: int = 32
    units: int = 64
    states: int = 256

    @property
    def variables(self) -> int:
        return self.height * self.width

    @property
    def fold_counts(self) -> list[int]:
        """Folds of each sum level: V, V/2, ..., 2."""
        counts, f = [], self.variables
        while f >= 2:
            counts.append(f)
            f //= 2
        return counts

    def parameter_shapes(self) -> dict[str, list[tuple[int, ...]]]:
        k = self.units
        return {
            "categorical": [(self.variables, self.states, k)],
            "levels": [(f, k, k) for f in self.fold_counts],
            "root": [(1, k)],
        }

    def init_parameters(self, generator: torch.Generator, device: torch.device | str = "cpu") -> dict[str, object]:
        """N(0, 1) logits for every parameter, drawn in a fixed order."""
        shapes = self.parameter_shapes()
        categorical = torch.randn(shapes["categorical"][0], generator=generator)
        levels = [torch.randn(s, generator=generator) for s in shapes["levels"]]
        root = torch.randn(shapes["root"][0], generator=generator)
        return {
            "categorical": categorical.to(device),
            "levels": [t.to(device) for t in levels],
            "root": root.to(device),
            "var_of_fold": torch.tensor(quad_tree_leaf_order(self.height, self.width), dtype=torch.int32).to(device),
        }

    def flops_per_sample(self) -> int:
        """Algorithmic FLOPs of the sum layers per sample (2 per multiply-add)."""
        k = self.units
        return 2 * k * k * sum(self.fold_counts) + 2 * k

    def hbm_bytes_per_sample(self, state_table: bool = False) -> int:
        """HBM bytes per sample that the layer kernels must move.

        Per sample: level 0 reads the sample's V uint8 pixels (its categorical
        log-probability rows come from a table that stays in L2) and writes
        (V, K); level l >= 1 reads the previous output (2F_l, K), the two
        Hadamard halves, and writes (F_l, K); the root reads (2, K) and
        writes one value.  fp32 values.  With the state table, level 0 is not
        written per sample and level 1 reads its rows from the table (L2):
        the sample's bytes are its pixels and levels 1 and up, less level 1's
        reads.
        """
        k = self.units
        counts = self.fold_counts
        elements = 0 if state_table else counts[0] * k  # level 0 output
        for level, f in enumerate(counts[1:], start=1):
            elements += (0 if state_table and level == 1 else 2 * f * k) + f * k
        elements += 2 * k + 1
        return 4 * elements + self.variables

    def uses_state_table(self, batch: int) -> bool:
        """Whether the first layer runs over the states (cheaper once the batch reaches half of them)."""
        return 2 * batch >= self.states and len(self.fold_counts) >= 2


class CircuitForward:
    """Forward pass of a QuadTreeCircuit on the current CUDA device.

    With gradients enabled and the state table in use (and K = 64), the call is one autograd node
    whose backward runs the fused layer backward kernels (xe_cp_layer_backward and friends);
    ``fused_backward=False`` keeps the per-operation backward of each call instead.
    """

    def __init__(self, circuit: QuadTreeCircuit, parameters: dict[str, object], shift: str = "max",
                 fused_backward: bool = True) -> None:
        self.circuit = circuit
        self.shift = shift
        self.fused_backward = fused_backward
        self.categorical = parameters["categorical"]
        self.levels = list(parameters["levels"])
        self.root = parameters["root"]
        self.var_of_fold = parameters["var_of_fold"]
        ops._check_tensors("CircuitForward", self.categorical, *self.levels, self.root)

    def __call__(self, pixels: torch.Tensor) -> torch.Tensor:
        """Log-likelihoods (B, 1) of uint8 pixels (B, variables)."""
        params = (self.categorical, self.root, *self.levels)
        if (self.fused_backward and ops._needs_grad(*params) and self.circuit.uses_state_table(pixels.shape[0])
                and self.circuit.units == 64 and self.circuit.states <= 256):
            return _CircuitFunction.apply(self, pixels, *params)
        table = ops.softmax(self.categorical, 1, log_output=True)
        state_table = self.circuit.uses_state_table(pixels.shape[0])
        y = None
        for level, logits in enumerate(self.levels):
            w = ops.softmax(logits, 2)  # (F, O, K) linear weights
            b_op = w.permute(0, 2, 1)  # (F, K, O), k contiguous
            if level == 0 and state_table:
                # the first sum layer for every state of each variable: (F0, states, K)
                y = ops.logspace_gemm(table, b_op, b_linear=True, shift=self.shift)
            elif level == 0:
                # the categorical gather is fused into the first sum layer's A rows
                y = ops.logspace_gemm_gather(table, pixels, self.var_of_fold, b_op, b_linear=True, shift=self.shift)
            elif level == 1 and state_table:
                # both Hadamard halves gathered from the state table
                y = ops.logspace_gemm_gather_pair(y, pixels, self.var_of_fold, b_op, b_linear=True, shift=self.shift)
            else:
                half = y.shape[0] // 2
                y = ops.logspace_gemm(y[:half], b_op, a2=y[half:], b_linear=True, shift=self.shift)
        w_root = ops.softmax(self.root, 1)  # (1, K)
        b_root = w_root.t().unsqueeze(0)  # (1, K, 1)
        ll = ops.logspace_gemm(y[0:1], b_root, a2=y[1:2], b_linear=True, shift=self.shift)
        return ll[0]


def _softmax_grad(y: torch.Tensor, dy: torch.Tensor, axis: int) -> torch.Tensor:
    """dx of y = softmax(x) over ``axis``: y (dy - sum(dy y))."""
    dot = ops.reduce(ops.elementwise("mul", dy, y), (axis,), "sum", keepdims=True)
    return ops.elementwise("mul", y, ops.elementwise("sub", dy, dot))


class _CircuitFunction(torch.autograd.Function):
    """The state-table forward of CircuitForward as one autograd node.

    Backward, from the root down (the shifts are stop_gradients, translate.py:727-740):
      root        elementwise: r = G exp(h - ll) for h the sum of the two top halves, dh = r w_root,
                  dw_root = sum_b r;
      levels >= 2 xe_cp_layer_backward: dA of both halves and dw from one pass over the layer's
                  input halves, output and gradient, the gradient of level l's output being
                  level l+1's dA read for both halves (fold f reads f mod F_{l+1});
      level 1     xe_cp_layer_backward_gather_pair over the state table, then
                  xe_state_table_pair_grad: the gradient of the table;
      level 0     xe_cp_layer_backward over the categorical log-table (M = states);
      parameters  the softmax / log-softmax backward of the weights and the categorical logits.
    """

    @staticmethod
    def forward(ctx, fwd: "CircuitForward", pixels, categorical, root, *levels):
        shift = fwd.shift
        table = ops.softmax(categorical, 1, log_output=True)
        weights = [ops.softmax(logits, 2) for logits in levels]
        ys = [ops.logspace_gemm(table, weights[0].permute(0, 2, 1), b_linear=True, shift=shift)]
        ys.append(ops.logspace_gemm_gather_pair(ys[0], pixels, fwd.var_of_fold, weights[1].permute(0, 2, 1),
                                                b_linear=True, shift=shift))
        for w in weights[2:]:
            y = ys[-1]
            half = y.shape[0] // 2
            ys.append(ops.logspace_gemm(y[:half], w.permute(0, 2, 1), a2=y[half:], b_linear=True, shift=shift))
        w_root = ops.softmax(root, 1)
        b_root = w_root.t().unsqueeze(0)
        top = ys[-1]
        ll = ops.logspace_gemm(top[0:1], b_root, a2=top[1:2], b_linear=True, shift=shift)
        ctx.fwd = fwd
        ctx.save_for_backward(pixels, table, w_root, ll, *weights, *ys)
        ctx.n_levels = len(levels)
        return ll[0]

    @staticmethod
    def backward(ctx, g_ll):
        fwd = ctx.fwd
        shift = fwd.shift
        saved = ctx.saved_tensors
        pixels, table, w_root, ll = saved[:4]
        n = ctx.n_levels
        weights, ys = saved[4:4 + n], saved[4 + n:]
        top = ys[-1]
        # root: ll[b] = log sum_k exp(h[b,k]) w[k] (shifted), h = top[0] + top[1]; with
        # r[b,k] = g[b] exp(h[b,k] - ll[b]): dh = r * w, dw = sum_b r
        h = ops.elementwise("add", top[0], top[1])
        r = ops.elementwise("rescale", g_ll.contiguous(), h, ll[0])
        d_root = _softmax_grad(w_root, ops.reduce(r, (0,), "sum", keepdims=True), 1)
        g = ops.elementwise("mul", r, w_root).unsqueeze(0)  # (1, B, K): the gradient of both top halves
        d_levels = [None] * n
        for level in range(n - 1, 1, -1):
            y_in = ys[level - 1]
            half = y_in.shape[0] // 2
            g, dw = ops.cp_layer_backward(y_in[:half], ys[level], g, weights[level], a2=y_in[half:], shift=shift)
            d_levels[level] = _softmax_grad(weights[level], dw, 2)
        # the pixels variable-major (strides (1, batch)): 32 samples' values of a variable in one sector
        pixels_vm = ops.variable_major(pixels)
        g, dw = ops.cp_layer_backward_gather_pair(ys[0], pixels_vm, fwd.var_of_fold, ys[1], g, weights[1], shift=shift)
        d_levels[1] = _softmax_grad(weights[1], dw, 2)
        g = ops.state_table_pair_grad(g, pixels_vm, fwd.var_of_fold, table.shape[1])
        d_table, dw = ops.cp_layer_backward(table, ys[0], g, weights[0], shift=shift)
        d_levels[0] = _softmax_grad(weights[0], dw, 2)
        total = ops.reduce(d_table, (1,), "sum", keepdims=True)
        d_categorical = ops.elementwise("sub", d_table, ops.elementwise("mul_exp", total, table))
        return None, None, d_categorical, d_root, *d_levels


def demo_circuit_program(xe, height: int, width: int, units: int, batch: int, stability_mode: str = "logspace_max",
                         layer: str = "cp"):
    """The demo's folded quad-tree circuit program, built and folded by the reference package ``xe``.

    The expression is the one demo/cirkit.py:131-210 builds from a cirkit quad-tree circuit
    (cirkit is not needed): leaf v is ``xe.select(data, v)`` of the (variables, batch, units)
    categorical probabilities, and the root has one output unit under ``xe.log``.  The two children
    of a region (the pairing of quad_tree_leaf_order) are joined
    * ``layer="cp"`` (--sum-product-layer cp): by the Hadamard product 'ab,ab->ab' of their sum
      layers 'ab,cb->ac', softmax(Parameter) weights over the input units;
    * ``layer="tucker"`` (--sum-product-layer tucker): by the Kronecker product 'ab,ac->abc'
      followed by the sum layer 'abc,dbc->ad' over the unit pairs, weights softmaxed over both.
    It is folded as demo/cirkit.py:478-479 folds it: FoldSameShapedOperations, then
    OptimizeContractionPaths (preprocess.py), which fuses each Kronecker product into its sum
    layer ('acde,abd,abe->abc').  Returns the folded RichProgram and the index of its data input;
    every other input is a packed parameter.
    """
    if layer not in ("cp", "tucker"):
        raise ValueError(f"unknown sum-product layer {layer!r}; expected 'cp' or 'tucker'")
    tensor_expression = importlib.import_module(xe.__name__ + ".interface.tensor_expression")
    preprocess = importlib.import_module(xe.__name__ + ".preprocess")
    parameter = tensor_expression.Parameter
    variables = height * width
    data = xe.array(torch.empty((variables, batch, units), dtype=torch.float32))

    def sum_layer(child, outputs: int = units):
        weights = xe.softmax(parameter(xe.array(torch.empty((outputs, units), dtype=torch.float32))), axis=1)
        return xe.einsum("ab,cb->ac", child, weights)

    def tucker_layer(left, right, outputs: int = units):
        weights = xe.softmax(parameter(xe.array(torch.empty((outputs, units, units), dtype=torch.float32))), axis=(1, 2))
        return xe.einsum("abc,dbc->ad", xe.einsum("ab,ac->abc", left, right), weights)

    if layer == "cp":
        level = [sum_layer(xe.select(data, v)) for v in quad_tree_leaf_order(height, width)]
        while len(level) > 2:
            half = len(level) // 2
            level = [sum_layer(xe.einsum("ab,ab->ab", level[i], level[i + half])) for i in range(half)]
        root = sum_layer(xe.einsum("ab,ab->ab", level[0], level[1]), outputs=1)
    else:
        level = [xe.select(data, v) for v in quad_tree_leaf_order(height, width)]
        while len(level) > 2:
            half = len(level) // 2
            level = [tucker_layer(level[i], level[i + half]) for i in range(half)]
        root = tucker_layer(level[0], level[1], outputs=1)
    program, _ = xe.extract_program(xe.log(root), stability_mode=stability_mode)
    folded = preprocess.FoldSameShapedOperations.apply_with_metadata(program)
    folded_program = preprocess.OptimizeContractionPaths.apply(folded.program)
    data_inputs = [i for i in range(folded_program.n_inputs) if i not in folded_program.parameter_indices]
    if len(data_inputs) != 1:
        raise ValueError(f"expected one data input in the folded circuit, found {len(data_inputs)}")
    return folded_program, data_inputs[0]


def demo_circuit_inputs(program, data_input: int, generator: torch.Generator, device: torch.device | str = "cpu"):
    """Seeded inputs of a demo_circuit_program: the data input holds categorical probabilities
    (softmax over the units of N(0, 1) logits, a stand-in for the gathered state rows), every
    parameter N(0, 1) logits, as the demo initialises them (demo/cirkit.py:511-518)."""
    inputs = []
    for i in range(program.n_inputs):
        shape = tuple(program.shapes[i])
        values = torch.randn(shape, generator=generator, device=generator.device)
        inputs.append((torch.softmax(values, dim=-1) if i == data_input else values).to(device))
    return inputs
