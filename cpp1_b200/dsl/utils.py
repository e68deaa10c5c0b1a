"""Graph utilities of the DSL (same names as the reference's src/dsl/utils.py)."""
from __future__ import annotations

from .matrix import Matrix
from .operations import Operation
from .var import Var


def var_names(self, frame_locals):
    """Name every unnamed Matrix in ``frame_locals`` after its variable."""
    for name, var in frame_locals.items():
        if isinstance(var, Matrix) and (getattr(var, "name", None) in (None, "unnamed")):
            var.name = name


def _all_operations(output_nodes):
    seen, found, stack = set(), set(), list(output_nodes)
    while stack:
        node = stack.pop()
        if id(node) in seen:
            continue
        seen.add(id(node))
        if isinstance(node, Operation):
            found.add(node)
            stack.extend(node.operands)
    return found


def topological_sort_operations(output_nodes):
    """Operations reachable from ``output_nodes``, every operand before its
    consumer; ties broken by operation name.  Raises on a cycle."""
    done, active, order = set(), set(), []

    def visit(node):
        if id(node) in active:
            raise ValueError("Cycle detected in the DSL graph. ")
        if id(node) in done:
            return
        active.add(id(node))
        if isinstance(node, Operation):
            for child in node.operands:
                visit(child)
        active.discard(id(node))
        done.add(id(node))
        if isinstance(node, Operation):
            order.append(node)

    for op in sorted(_all_operations(output_nodes), key=lambda o: o.name or str(id(o))):
        visit(op)
    return order


def get_graph_io(output_nodes):
    """(input matrices sorted by name, symbolic dimension Vars sorted by name)."""
    inputs, dims, seen, stack = {}, {}, set(), list(output_nodes)
    while stack:
        node = stack.pop()
        if id(node) in seen:
            continue
        seen.add(id(node))
        for d in getattr(node, "shape", ()):
            if isinstance(d, Var):
                dims.setdefault(str(d.name), d)
        if isinstance(node, Operation):
            stack.extend(node.operands)
        elif isinstance(node, Matrix):
            inputs[id(node)] = node
    mats = sorted(inputs.values(), key=lambda m: m.name or "")
    return mats, [dims[k] for k in sorted(dims)]
