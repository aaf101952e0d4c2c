"""Canonical text dump of the reference's IR -- TEST INFRASTRUCTURE ONLY.

Runs inside the reference worker processes (oracle/ref_runner.py) on the
reference's own IR objects (opencuda/ir/nodes.py:23-289) and prints them in
the same line format as the GPU parser's IR dump, so the two compare as bytes:

    kernel <name> next_id=<n>
     launch <bounds...>                (when __launch_bounds__ was given)
     param <name> <ty>
     shared <name> <ty> <count>
     local <name> <ty> <count> <value>
     block <label>
      <value> = bin <op> <a>, <b>
      <value> = cmp <op> <a>, <b>
      <value> = select <c>, <a>, <b>
      <value> = load <addr>
      store <addr>, <value>
      <value> = cvt <src>
      <value|_> = call <func>(<args>)
      <value> = param <index> <name>
      term ret [<operand>] | term br <label> | term cbr <c>, <t>, <f>

Values print as %<id>:<name>:<ty>; constants as #<ty>:i:<int> or
#<ty>:f:<IEEE-754 double bits in hex> (the reference keeps Python ints and
floats apart even under a float type); symbols as @<name>.  Types print as
the scalar's C name or ptr(<pointee>,<addr space>,<volatile 0/1>).
"""
from __future__ import annotations

import struct


def ty_str(t) -> str:
    from opencuda.ir.types import ScalarTy, PtrTy
    if isinstance(t, ScalarTy):
        return t.scalar.value
    if isinstance(t, PtrTy):
        asp = t.addr_space.value if hasattr(t.addr_space, "value") else str(t.addr_space)
        return f"ptr({ty_str(t.pointee)},{asp},{1 if t.volatile else 0})"
    if type(t).__name__ == "StructTy":
        return f"struct({t.name})"
    return f"?{type(t).__name__}"


def op_str(o) -> str:
    from opencuda.ir.nodes import Value, Const, SymbolRef
    if o is None:
        return "_"
    if isinstance(o, Value):
        return f"%{o.id}:{o.name}:{ty_str(o.ty)}"
    if isinstance(o, Const):
        v = o.value
        if isinstance(v, bool):
            v = int(v)
        if isinstance(v, float):
            bits = struct.unpack(">Q", struct.pack(">d", v))[0]
            return f"#{ty_str(o.ty)}:f:{bits:016x}"
        return f"#{ty_str(o.ty)}:i:{int(v)}"
    if isinstance(o, SymbolRef):
        return f"@{o.sym_name}"
    return f"?{type(o).__name__}"


def inst_str(i) -> str:
    from opencuda.ir import nodes as N
    if isinstance(i, N.BinInst):
        return f"{op_str(i.dest)} = bin {i.op.value} {op_str(i.lhs)}, {op_str(i.rhs)}"
    if isinstance(i, N.CmpInst):
        return f"{op_str(i.dest)} = cmp {i.op.value} {op_str(i.lhs)}, {op_str(i.rhs)}"
    if isinstance(i, N.SelectInst):
        return (f"{op_str(i.dest)} = select {op_str(i.cond)}, {op_str(i.true_val)}, "
                f"{op_str(i.false_val)}")
    if isinstance(i, N.LoadInst):
        return f"{op_str(i.dest)} = load {op_str(i.addr)}"
    if isinstance(i, N.StoreInst):
        return f"store {op_str(i.addr)}, {op_str(i.value)}"
    if isinstance(i, N.CvtInst):
        return f"{op_str(i.dest)} = cvt {op_str(i.src)}"
    if isinstance(i, N.CallInst):
        return f"{op_str(i.dest)} = call {i.func}({', '.join(op_str(a) for a in i.args)})"
    if isinstance(i, N.GlobalAddrInst):
        asp = i.addr_space.value if hasattr(i.addr_space, "value") else str(i.addr_space)
        return f"{op_str(i.dest)} = gaddr @{i.sym_name} {asp}"
    if isinstance(i, N.ParamInst):
        return f"{op_str(i.dest)} = param {i.param_index} {i.param_name}"
    if isinstance(i, N.PrintfInst):
        fmt = i.fmt.encode("utf-8", "surrogateescape").hex()
        return f"printf {fmt}({', '.join(op_str(a) for a in i.args)})"
    if isinstance(i, N.AsmInst):
        tmpl = i.template.encode("utf-8", "surrogateescape").hex()
        outs = ', '.join(op_str(v) for _, v in i.outputs)
        ins = ', '.join(op_str(v) for _, v in i.inputs)
        return f"asm {tmpl}({outs}; {ins})"
    return f"?{type(i).__name__}"


def term_str(t) -> str:
    from opencuda.ir import nodes as N
    if t is None:
        return "term none"
    if isinstance(t, N.RetTerm):
        return "term ret" + ("" if t.ret_val is None else " " + op_str(t.ret_val))
    if isinstance(t, N.BrTerm):
        return f"term br {t.target}"
    if isinstance(t, N.CondBrTerm):
        return f"term cbr {op_str(t.cond)}, {t.true_bb}, {t.false_bb}"
    return f"term ?{type(t).__name__}"


def dump_kernel(k) -> str:
    out = [f"kernel {k.name} next_id={k._next_id}"]
    lb = getattr(k, "_launch_bounds", None)
    if lb:
        out.append(" launch " + " ".join(str(x) for x in lb))
    for p in k.params:
        out.append(f" param {p.name} {ty_str(p.ty)}")
    for name, ty, count in getattr(k, "_shared_decls", []) or []:
        out.append(f" shared {name} {ty_str(ty)} {count}")
    for name, ty, count, val in getattr(k, "_local_decls", []) or []:
        out.append(f" local {name} {ty_str(ty)} {count} {op_str(val)}")
    for b in k.blocks:
        out.append(f" block {b.label}")
        for i in b.instructions:
            out.append("  " + inst_str(i))
        out.append("  " + term_str(b.terminator))
    return "\n".join(out)


def dump_module(m) -> str:
    parts = [dump_kernel(k) for k in m.kernels]
    if m.device_functions or m.global_vars:
        parts.append("module-extras")
    return "\n".join(parts) + "\n"


def verify_text(module, check_reachability: bool) -> str:
    """verify_module(module, check_reachability) (opencuda/ir/verify_ir.py:302)
    as text: per kernel with violations, `kernel <name>` then its error
    strings, one per line -- the GPU verifier's output format."""
    from opencuda.ir.verify_ir import verify_module
    out = []
    for name, errs in verify_module(module, check_reachability=check_reachability).items():
        out.append(f"kernel {name}\n")
        out.extend(e + "\n" for e in errs)
    return "".join(out)
