"""Multi-solution curriculum: alternative solutions of code and math tasks that are equivalent by
construction (reference src/omnicoder/tools/multi_solution_gen.py:1-127, which renames short
variable names by regular expression -- a rename that can collide with other names or touch
strings -- and appends comments suggesting recursion / iteration rewrites).

Code (Python):
  rename_locals    every local variable of every function that is not a parameter, a global /
                   nonlocal name, an import / exception / match binding or a name a nested scope
                   touches gets a fresh name
                   (`v0`, `v1`, ... not used anywhere in the module), through the AST, so strings,
                   attributes, keyword arguments and other scopes are untouched
  canonical        the AST printed back (uniform formatting, comments dropped)
  When the row has tests, each variant runs against them in the sandbox and is kept only if it
  passes as the original does.
Math (sympy):
  for every `lhs = rhs` line of the solution: the equation moved to one side and expanded
  (`lhs - rhs = 0`), factored, and, with one unknown, solved; each is checked to have the
  original equation's solution set.  sympy parses the text by evaluating it, so the input is
  expected to be the user's own data.
"""
from __future__ import annotations

import argparse
import ast
import json
import os


class _Renamer(ast.NodeTransformer):
    def __init__(self, mapping: dict):
        self.mapping = mapping

    def visit_Name(self, node: ast.Name):
        if node.id in self.mapping:
            return ast.copy_location(ast.Name(id=self.mapping[node.id], ctx=node.ctx), node)
        return node


def _local_names(fn: ast.FunctionDef) -> set:
    params = {a.arg for a in fn.args.args + fn.args.posonlyargs + fn.args.kwonlyargs}
    for a in (fn.args.vararg, fn.args.kwarg):
        if a is not None:
            params.add(a.arg)
    declared, stored, nested = set(), set(), set()
    for node in ast.walk(fn):
        if isinstance(node, (ast.Global, ast.Nonlocal)):
            declared.update(node.names)
        elif isinstance(node, (ast.FunctionDef, ast.AsyncFunctionDef, ast.ClassDef, ast.Lambda)) and node is not fn:
            for sub in ast.walk(node):               # names a nested scope touches stay as they are
                if isinstance(sub, ast.Name):
                    nested.add(sub.id)
                elif isinstance(sub, ast.arg):
                    nested.add(sub.arg)
            if not isinstance(node, ast.Lambda):
                nested.add(node.name)
        elif isinstance(node, ast.Name) and isinstance(node.ctx, ast.Store):
            stored.add(node.id)
        elif isinstance(node, ast.ExceptHandler) and node.name:      # bound by name strings, not Name nodes
            declared.add(node.name)
        elif isinstance(node, (ast.Import, ast.ImportFrom)):
            declared.update((al.asname or al.name).split(".")[0] for al in node.names)
        elif isinstance(node, (ast.MatchAs, ast.MatchStar)) and node.name:
            declared.add(node.name)
        elif isinstance(node, ast.MatchMapping) and node.rest:
            declared.add(node.rest)
    return stored - params - declared - nested


def rename_locals(src: str) -> str:
    tree = ast.parse(src)
    used = {n.id for n in ast.walk(tree) if isinstance(n, ast.Name)} | \
        {n.arg for n in ast.walk(tree) if isinstance(n, ast.arg)} | \
        {n.name for n in ast.walk(tree) if isinstance(n, (ast.FunctionDef, ast.AsyncFunctionDef, ast.ClassDef))}
    counter = 0
    for fn in [n for n in ast.walk(tree) if isinstance(n, (ast.FunctionDef, ast.AsyncFunctionDef))]:
        mapping = {}
        for name in sorted(_local_names(fn)):
            while f"v{counter}" in used:
                counter += 1
            mapping[name] = f"v{counter}"
            used.add(mapping[name])
        if mapping:
            for i, stmt in enumerate(fn.body):
                fn.body[i] = _Renamer(mapping).visit(stmt)
    return ast.unparse(ast.fix_missing_locations(tree))


def canonical(src: str) -> str:
    return ast.unparse(ast.parse(src))


def code_variants(solution: str, tests: str | None = None, timeout: int = 30) -> list[dict]:
    from ..sfb.sandbox import verify_with_tests
    out = []
    for name, fn in (("rename_locals", rename_locals), ("canonical", canonical)):
        try:
            alt = fn(solution)
        except SyntaxError:
            return []
        if alt.strip() == solution.strip():
            continue
        rec = {"variant": name, "code": alt}
        if tests:
            rec["verified"] = verify_with_tests(alt, tests, timeout=timeout).ok
        out.append(rec)
    return out


def math_variants(solution: str) -> list[dict]:
    import sympy as sp
    out = []
    for line in solution.splitlines():
        if line.count("=") != 1 or any(op in line for op in ("==", "<=", ">=", "!=")):
            continue
        lhs, rhs = line.split("=")
        try:
            eq = sp.sympify(lhs) - sp.sympify(rhs)
        except (sp.SympifyError, SyntaxError, TypeError):
            continue
        free = sorted(eq.free_symbols, key=str)
        if not free:
            continue
        base = set(sp.solve(eq, free[0])) if len(free) == 1 else None
        cands = [("one_side_expanded", f"{sp.expand(eq)} = 0"), ("factored", f"{sp.factor(eq)} = 0")]
        if len(free) == 1:
            cands.append(("solved", ", ".join(f"{free[0]} = {s}" for s in sorted(base, key=str))))
        for name, text in cands:
            ok = True
            if base is not None and name != "solved":
                ok = set(sp.solve(sp.sympify(text.split("=")[0]), free[0])) == base
            out.append({"variant": name, "solution": text, "verified": ok, "from": line.strip()})
    return out


def main(argv=None):
    ap = argparse.ArgumentParser(description="equivalent alternative solutions of code / math tasks")
    ap.add_argument("--input", required=True)
    ap.add_argument("--domain", required=True, choices=["code", "math"])
    ap.add_argument("--out", required=True)
    ap.add_argument("--keep_unverified", action="store_true")
    a = ap.parse_args(argv)
    out = []
    with open(a.input, encoding="utf-8") as f:
        rows = [json.loads(ln) for ln in f if ln.strip()]
    for r in rows:
        if a.domain == "code":
            sol = str(r.get("target") or r.get("solution") or r.get("code") or "")
            for v in code_variants(sol, r.get("tests")):
                if v.get("verified", True) or a.keep_unverified:
                    out.append({"prompt": r.get("prompt") or r.get("question") or "", "targets": [sol],
                                "variant": v["variant"], "alt_code": v["code"], "verified": v.get("verified")})
        else:
            sol = str(r.get("answer") or r.get("solution") or "")
            for v in math_variants(sol):
                if v["verified"] or a.keep_unverified:
                    out.append({"question": r.get("question") or r.get("problem") or "", "answer": sol,
                                "variant": v["variant"], "alt_solution": v["solution"], "verified": v["verified"]})
    os.makedirs(os.path.dirname(a.out) or ".", exist_ok=True)
    with open(a.out, "w", encoding="utf-8") as f:
        f.write("\n".join(json.dumps(o, ensure_ascii=False) for o in out) + ("\n" if out else ""))
    print(json.dumps({"rows": len(rows), "wrote": len(out), "out": a.out}))
    return 0


if __name__ == "__main__":
    main()
