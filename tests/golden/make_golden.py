"""Generates the golden vectors that pin the oracle and the B200 path.

Runs the REFERENCE implementation (extended_einsum, imported from its source
tree) on seeded inputs and records inputs and outputs:

* fp32 results of the reference's own torch executor
  (translate_to_backend_program + TorchBackendFunctions + run_program), the
  configuration the B200 path must match;
* fp64 results of the reference's numpy executor, as ground truth;

in every stable mode the reference accepts for the program (logspace_max,
logspace_min, scaled_sum, scaled_max, scaled_min; a mode the reference
rejects is noted under "rejected"), and for a few programs the fp64
gradients of sum(out * w) for a fixed seeded w (the reference's torch executor
through autograd, shifts detached as it detaches them).

Cases: small instances of every hot-path pattern (log-space matmul, batched
matmul with N(0, 8^2) values, folded CP sum layer, Tucker layer, softmax, a
folded quad-tree circuit), plus the reference's own known-answer and
mode-agreement programs (tests/test_backend_translation.py of the reference).

Usage (needs the reference source tree; the outputs are committed):
    python tests/golden/make_golden.py /path/to/extended_einsum
"""

from __future__ import annotations

import json
import math
import sys
from pathlib import Path

import numpy as np
import torch

OUT_DIR = Path(__file__).resolve().parent
ALL_MODES = ("logspace_max", "logspace_min", "scaled_sum", "scaled_max", "scaled_min")
# programs whose gradients (of sum(out * w), fixed w) are recorded, logspace_max, fp64
GRAD_PROGRAMS = ("matmul_logu", "batched_n64", "cp_layer", "softmax_rows", "tucker", "tucker_two_levels", "mixing_layer",
                 "agreement_add", "circuit_4x4")


def main(reference_root: str) -> None:
    sys.path.insert(0, str(Path(reference_root) / "src"))
    sys.path.insert(0, str(Path(reference_root)))
    import extended_einsum as xe
    from extended_einsum.backend_translation.runtime import run_program
    from extended_einsum.backend_translation.translate import translate_to_backend_program
    from extended_einsum.backends.numpy import NumpyBackendFunctions
    from extended_einsum.backends.torch import TorchBackendFunctions
    from extended_einsum.interface.tensor_expression import Parameter
    from extended_einsum.language import rich_operators as ro
    from extended_einsum.language.rich_instruction import RichInstruction
    from extended_einsum.language.rich_program import RichProgram

    arrays: dict[str, np.ndarray] = {}
    programs: dict[str, dict] = {}

    def serialize(program) -> dict:
        instructions = []
        for ins in program.instructions:
            op = ins.operator
            attrs = {}
            for attr in ("axis", "index", "start", "stop", "format_string"):
                if hasattr(op, attr):
                    value = getattr(op, attr)
                    attrs[attr] = list(value) if isinstance(value, tuple) else value
            instructions.append([op.name, attrs, list(ins.argument_ssa_ids)])
        return {
            "n_inputs": program.n_inputs,
            "parameter_indices": sorted(program.parameter_indices),
            "shapes": [list(s) for s in program.shapes],
            "instructions": instructions,
        }

    def with_mode(program, mode):
        return RichProgram(
            instructions=program.instructions,
            n_inputs=program.n_inputs,
            stability_mode=mode,
            tensor_formats=program.tensor_formats,
            shapes=program.shapes,
            parameter_indices=program.parameter_indices,
        )

    def run_reference(program, inputs: list[np.ndarray]) -> tuple[np.ndarray, np.ndarray]:
        torch_inputs = [torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)) if x.dtype.kind == "f" else torch.from_numpy(x) for x in inputs]
        out32 = run_program(translate_to_backend_program(program, TorchBackendFunctions()), torch_inputs).numpy()
        # the fp64 ground truth is computed from the same fp32-rounded inputs that are stored
        np_inputs = [x.astype(np.float32).astype(np.float64) if x.dtype.kind == "f" else x for x in inputs]
        out64 = run_program(translate_to_backend_program(program, NumpyBackendFunctions()), np_inputs)
        return np.asarray(out32), np.asarray(out64)

    def reference_grads(program, inputs: list[np.ndarray], seed: int):
        """Gradients of sum(out * w) through the reference's torch executor, in fp64."""
        tins = [torch.from_numpy(x.astype(np.float32).astype(np.float64)).requires_grad_(True) for x in inputs]
        out = run_program(translate_to_backend_program(program, TorchBackendFunctions()), tins)
        w = np.random.default_rng(seed).standard_normal(tuple(out.shape)).astype(np.float32)
        (out * torch.from_numpy(w.astype(np.float64))).sum().backward()
        return w, [t.grad.numpy() if t.grad is not None else None for t in tins]

    def record(name: str, program, inputs: list[np.ndarray], modes=ALL_MODES) -> None:
        programs[name] = serialize(program)
        for i, x in enumerate(inputs):
            arrays[f"{name}/in{i}"] = x.astype(np.float32) if x.dtype.kind == "f" else x
        recorded = []
        for mode in modes:
            try:
                out32, out64 = run_reference(with_mode(program, mode), inputs)
            except Exception as error:  # noqa: BLE001 - a mode the reference rejects for this program
                if mode.startswith("logspace"):
                    raise
                programs[name].setdefault("rejected", {})[mode] = f"{type(error).__name__}: {error}"[:200]
                continue
            arrays[f"{name}/{mode}/f32"] = out32
            arrays[f"{name}/{mode}/f64"] = out64
            recorded.append(mode)
            if mode == "logspace_max" and name in GRAD_PROGRAMS:
                w, grads = reference_grads(with_mode(program, mode), inputs, seed=len(name))
                arrays[f"{name}/{mode}/grad_weights"] = w
                for i, grad in enumerate(grads):
                    if grad is not None:
                        arrays[f"{name}/{mode}/grad{i}"] = grad
        programs[name]["modes"] = recorded

    # -- hot-path patterns through the public expression API ------------------
    torch.manual_seed(0)
    a = torch.log(torch.rand(64, 96))
    b = torch.log(torch.rand(96, 80))
    prog, _ = xe.extract_program(xe.log(xe.einsum("ik,kj->ij", xe.exp(xe.array(a)), xe.exp(xe.array(b)))), "logspace_max")
    record("matmul_logu", prog, [a.numpy(), b.numpy()])

    torch.manual_seed(1)
    a = 8.0 * torch.randn(3, 40, 72)
    b = 8.0 * torch.randn(3, 72, 56)
    prog, _ = xe.extract_program(xe.log(xe.einsum("bik,bkj->bij", xe.exp(xe.array(a)), xe.exp(xe.array(b)))), "logspace_max")
    record("batched_n64", prog, [a.numpy(), b.numpy()])

    torch.manual_seed(2)
    left = torch.randn(20, 3, 32) - 3.0
    right = torch.randn(20, 3, 32) - 3.0
    w_logits = torch.randn(3, 8, 32, 32)
    expr = xe.log(
        xe.einsum(
            "bfi,bfj,foij->bfo",
            xe.exp(xe.array(left)),
            xe.exp(xe.array(right)),
            xe.softmax(Parameter(xe.array(w_logits)), axis=(2, 3)),
        )
    )
    prog, _ = xe.extract_program(expr, "logspace_max")
    record("tucker", prog, [left.numpy(), right.numpy(), w_logits.numpy()])

    torch.manual_seed(3)
    x = torch.randn(4, 24, 16) - 2.0
    w_logits = torch.randn(4, 16, 16)
    expr = xe.log(xe.einsum("dac,dbc->dab", xe.exp(xe.array(x)), xe.softmax(Parameter(xe.array(w_logits)), axis=2)))
    prog, _ = xe.extract_program(expr, "logspace_max")
    record("cp_layer", prog, [x.numpy(), w_logits.numpy()])

    # mixing layer of the quad-graph circuits (the demo's 'bhu,uh->bu' over stacked children,
    # demo/cirkit.py:163-169) and a two-level Tucker circuit fragment
    torch.manual_seed(6)
    children = [torch.randn(48, 20) - 3.0 for _ in range(3)]
    mix_logits = torch.randn(20, 3)
    stacked = xe.stack([xe.exp(xe.array(ch)) for ch in children], axis=1)
    expr = xe.log(xe.einsum("bhu,uh->bu", stacked, xe.softmax(Parameter(xe.array(mix_logits)), axis=1)))
    prog, args = xe.extract_program(expr, "logspace_max")
    record("mixing_layer", prog, [a.backend_array.numpy() for a in args])

    torch.manual_seed(7)
    leaves = [torch.randn(12, 4, 32) - 3.0 for _ in range(3)]
    w1 = torch.randn(4, 32, 32, 32)
    w2 = torch.randn(4, 32, 32, 32)
    e = [xe.exp(xe.array(t)) for t in leaves]
    lvl1 = xe.einsum("bfi,bfj,foij->bfo", e[0], e[1], xe.softmax(Parameter(xe.array(w1)), axis=(2, 3)))
    expr = xe.log(xe.einsum("bfi,bfj,foij->bfo", lvl1, e[2], xe.softmax(Parameter(xe.array(w2)), axis=(2, 3))))
    prog, args = xe.extract_program(expr, "logspace_max")
    record("tucker_two_levels", prog, [a.backend_array.numpy() for a in args])

    torch.manual_seed(4)
    for name, shape, axis in (("softmax_rows", (6, 37), 1), ("softmax_block", (3, 5, 7), (1, 2)), ("softmax_mid", (4, 9, 5), 1), ("softmax_wide", (3, 1500), 1)):
        x = 2.0 * torch.randn(*shape)
        prog, _ = xe.extract_program(xe.softmax(xe.array(x), axis=axis), "logspace_max")
        record(name, prog, [x.numpy()])

    # -- folded quad-tree circuits (structure of extended_einsum_b200.circuit) -
    def circuit_program(height: int, width: int, units: int, states: int, batch: int, seed: int):
        g = torch.Generator().manual_seed(seed)
        variables = height * width
        levels = int(math.log2(variables))
        cat_logits = torch.randn(variables, states, units, generator=g)
        level_logits = [torch.randn(variables >> l, units, units, generator=g) for l in range(levels)]
        root_logits = torch.randn(1, units, generator=g)
        pixels = torch.randint(states, (batch, variables), generator=g, dtype=torch.uint8)
        sys.path.insert(0, str(OUT_DIR.parents[1]))
        from extended_einsum_b200.circuit import quad_tree_leaf_order

        var_of_fold = torch.tensor(quad_tree_leaf_order(height, width), dtype=torch.int64)
        # the demo's categorical input (demo/cirkit.py:525-527), in fold order
        probs = torch.softmax(cat_logits, dim=1)
        data = probs[torch.arange(variables)[:, None], pixels[:, var_of_fold].T.long()].contiguous()
        # folded program: inputs 0 = data, 1..L = level logits, L+1 = root logits
        n_inputs = levels + 2
        instructions, shapes = [], [tuple(data.shape)] + [tuple(t.shape) for t in level_logits] + [tuple(root_logits.shape)]

        def add(op, args, shape):
            instructions.append(RichInstruction(op, tuple(args)))
            shapes.append(tuple(shape))
            return n_inputs + len(instructions) - 1

        y = None
        for level in range(levels):
            f = variables >> level
            w = add(ro.OperatorSoftmax(2), [1 + level], (f, units, units))
            if level == 0:
                x_id = 0
            else:
                lhs = add(ro.OperatorSlice(0, f, 0), [y], (f, batch, units))
                rhs = add(ro.OperatorSlice(f, 2 * f, 0), [y], (f, batch, units))
                x_id = add(ro.OperatorEinsum("cab,cab->cab"), [lhs, rhs], (f, batch, units))
            y = add(ro.OperatorEinsum("dac,dbc->dab"), [x_id, w], (f, batch, units))
        s0 = add(ro.OperatorSelect(0, 0), [y], (batch, units))
        s1 = add(ro.OperatorSelect(0, 1), [y], (batch, units))
        h = add(ro.OperatorEinsum("ab,ab->ab"), [s0, s1], (batch, units))
        wr = add(ro.OperatorSoftmax(1), [levels + 1], (1, units))
        root = add(ro.OperatorEinsum("ab,cb->ac"), [h, wr], (batch, 1))
        add(ro.OperatorLog(), [root], (batch, 1))
        program = RichProgram(
            instructions=instructions,
            n_inputs=n_inputs,
            stability_mode="logspace_max",
            tensor_formats=["dense"] * len(shapes),
            shapes=shapes,
            parameter_indices=frozenset(range(1, n_inputs)),
        )
        inputs = [data.numpy()] + [t.numpy() for t in level_logits] + [root_logits.numpy()]
        extras = {"categorical_logits": cat_logits.numpy(), "pixels": pixels.numpy(), "var_of_fold": var_of_fold.numpy().astype(np.int32)}
        return program, inputs, extras

    for name, dims in (("circuit_4x4", (4, 4, 8, 16, 32, 5)), ("circuit_8x8", (8, 8, 16, 32, 48, 6))):
        program, inputs, extras = circuit_program(*dims)
        record(name, program, inputs)
        for key, value in extras.items():
            arrays[f"{name}/{key}"] = value
        programs[name]["circuit"] = dict(zip(("height", "width", "units", "states", "batch", "seed"), dims))

    # -- the reference's own known-answer and agreement programs ---------------
    from tests import test_backend_translation as ref_tests

    known = {
        "row_shift_minus1000": ([ref_tests.RichInstruction(ro.OperatorExp(), (0,)), RichInstruction(ro.OperatorEinsum("bi, io -> bo"), (2, 1)), RichInstruction(ro.OperatorLog(), (3,))],
                                [np.array([[0.0, -1.0], [-1000.0, -1001.0]]), np.array([[1.0, 2.0], [3.0, 4.0]])], {1}),
        "axis_reorder_minus1000": ([RichInstruction(ro.OperatorExp(), (0,)), RichInstruction(ro.OperatorEinsum("ib, io -> bo"), (2, 1)), RichInstruction(ro.OperatorLog(), (3,))],
                                   [np.array([[0.0, -1000.0], [-1.0, -1001.0]]), np.array([[1.0, 2.0], [3.0, 4.0]])], {1}),
        "softmax_params_linear": ([RichInstruction(ro.OperatorSoftmax(axis=0), (1,)), RichInstruction(ro.OperatorExp(), (0,)), RichInstruction(ro.OperatorEinsum("bi, io -> bo"), (3, 2)), RichInstruction(ro.OperatorLog(), (4,))],
                                  [np.array([[0.0, -1.0], [-1000.0, -1001.0]]), np.array([[1.0, 2.0], [3.0, 4.0]])], {1}),
        "hadamard_is_add": ([RichInstruction(ro.OperatorEinsum("ij,ij->ij"), (0, 1)), RichInstruction(ro.OperatorLog(), (2,))],
                            [ref_tests.POSITIVE_MATRIX, ref_tests.OTHER_POSITIVE_MATRIX], set()),
        "kronecker_is_broadcast_add": ([RichInstruction(ro.OperatorEinsum("bi,bj->bij"), (0, 1)), RichInstruction(ro.OperatorLog(), (2,))],
                                       [ref_tests.POSITIVE_MATRIX[:, :2], ref_tests.OTHER_POSITIVE_MATRIX[:, :3]], set()),
        "exp_log_free": ([RichInstruction(ro.OperatorExp(), (0,)), RichInstruction(ro.OperatorLog(), (1,))],
                         [800.0 + ref_tests.MATRIX], set()),
        "huge_chain_1e30": (ref_tests._huge_chain_program("logspace_max", ref_tests.N_HUGE_FACTORS).instructions,
                            [1.0e30 * f for f in ref_tests.RAW_CHAIN_FACTORS], set()),
    }
    for case_name, instructions, tensors in ref_tests.AGREEMENT_CASES:
        if case_name == "subtract-with-mixed-sign-result":
            continue  # logspace cannot represent the negative result (reference test skips it too)
        known[f"agreement_{case_name}"] = (instructions, tensors, set())
    for name, (instructions, tensors, params) in known.items():
        n = len(tensors)
        program = RichProgram(
            instructions=list(instructions),
            n_inputs=n,
            stability_mode="logspace_max",
            tensor_formats=["dense"] * (n + len(instructions)),
            shapes=[tuple(np.shape(t)) for t in tensors] + [()] * len(instructions),
            parameter_indices=frozenset(params),
        )
        record(name, program, [np.asarray(t) for t in tensors])

    np.savez_compressed(OUT_DIR / "golden.npz", **arrays)
    (OUT_DIR / "programs.json").write_text(json.dumps(programs, indent=1, sort_keys=True))
    print(f"wrote {len(programs)} programs, {len(arrays)} arrays")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "extended_einsum")
