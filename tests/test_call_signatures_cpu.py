"""Static check that keyword arguments of internal calls exist in the callee.

Every call inside ``d3d_b200`` whose callee can be resolved without running
anything -- a function defined in the same module, a function imported from
another ``d3d_b200`` module by name, or ``self.method`` defined on the
enclosing class -- must only pass keywords the callee declares (unless it
takes ``**kwargs``).  A misspelled keyword on a rarely taken path (a GPU
branch, an error path) would otherwise only fail when that path runs."""
import ast
import pathlib

ROOT = pathlib.Path(__file__).resolve().parents[1] / "d3d_b200"


def _module_name(path: pathlib.Path) -> str:
    rel = path.relative_to(ROOT.parent).with_suffix("")
    parts = list(rel.parts)
    if parts[-1] == "__init__":
        parts = parts[:-1]
    return ".".join(parts)


def _params(fn: ast.FunctionDef):
    a = fn.args
    names = {x.arg for x in a.posonlyargs + a.args + a.kwonlyargs}
    return names, a.kwarg is not None


def _index():
    mods = {}
    for path in ROOT.rglob("*.py"):
        tree = ast.parse(path.read_text(), str(path))
        funcs, classes = {}, {}
        for node in tree.body:
            if isinstance(node, (ast.FunctionDef, ast.AsyncFunctionDef)):
                funcs[node.name] = _params(node)
            elif isinstance(node, ast.ClassDef):
                classes[node.name] = {n.name: _params(n) for n in node.body
                                      if isinstance(n, (ast.FunctionDef, ast.AsyncFunctionDef))}
        mods[_module_name(path)] = (path, tree, funcs, classes)
    return mods


def _resolve_from(mod: str, level: int, name: str) -> str:
    if level == 0:
        return name
    base = mod.split(".")
    pkg = base[:-level] if not mod.endswith("__init__") else base[:len(base) - level + 1]
    return ".".join(pkg + ([name] if name else []))


def test_internal_keyword_calls_match_signatures():
    mods = _index()
    problems = []
    for mod, (path, tree, funcs, classes) in mods.items():
        is_pkg = path.name == "__init__.py"
        known = dict(funcs)
        for node in ast.walk(tree):
            if isinstance(node, ast.ImportFrom):
                src = _resolve_from(mod + (".__init__" if is_pkg else ""), node.level, node.module or "")
                if src in mods:
                    for a in node.names:
                        f = mods[src][2].get(a.name)
                        if f is not None:
                            known[a.asname or a.name] = f
        for cls in [n for n in tree.body if isinstance(n, ast.ClassDef)]:
            methods = classes[cls.name]
            for node in ast.walk(cls):
                if (isinstance(node, ast.Call) and isinstance(node.func, ast.Attribute)
                        and isinstance(node.func.value, ast.Name) and node.func.value.id == "self"
                        and node.func.attr in methods):
                    names, var = methods[node.func.attr]
                    for kw in node.keywords:
                        if kw.arg is not None and not var and kw.arg not in names:
                            problems.append(f"{path}:{node.lineno} self.{node.func.attr}(... {kw.arg}=)")
        for node in ast.walk(tree):
            if isinstance(node, ast.Call) and isinstance(node.func, ast.Name) and node.func.id in known:
                names, var = known[node.func.id]
                for kw in node.keywords:
                    if kw.arg is not None and not var and kw.arg not in names:
                        problems.append(f"{path}:{node.lineno} {node.func.id}(... {kw.arg}=)")
    assert not problems, "\n".join(problems)
    assert len(mods) > 40
