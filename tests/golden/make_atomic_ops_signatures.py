"""Record the signatures of the reference operators that
fluxvla_b200.atomic_ops and fluxvla_b200.attention_triton_ops replace (the
functions pi05_flowmatching_inference.py imports from fluxvla/ops/atomic_ops.py
and from fluxvla/ops/triton/attention_triton_ops.py) as a JSON fixture.

Run in a checkout that has the reference tree:
    python tests/golden/make_atomic_ops_signatures.py <fluxvla root>
The reference module is parsed with ``ast`` (not imported: it needs Triton
kernels and CUDA extensions)."""
import ast
import json
import os
import sys

root = sys.argv[1] if len(sys.argv) > 1 else '.'
src = open(os.path.join(root, 'fluxvla/ops/atomic_ops.py')).read()
tree = ast.parse(src)
inf = ast.parse(open(os.path.join(
    root, 'fluxvla/models/vlas/pi05_flowmatching_inference.py')).read())
wanted = set()
for node in ast.walk(inf):
    if isinstance(node, ast.ImportFrom) and node.module == 'fluxvla.ops.atomic_ops':
        wanted |= {a.name for a in node.names}
sigs = {}
for node in tree.body:
    if isinstance(node, ast.FunctionDef) and node.name in wanted:
        a = node.args
        names = [x.arg for x in a.args]
        defaults = [ast.literal_eval(d) for d in a.defaults]
        sigs[node.name] = {
            'args': names,
            'defaults': dict(zip(names[len(names) - len(defaults):], defaults)),
            'line': node.lineno}
# the Triton attention kernels pi05_flowmatching_inference.py launches itself
att = ast.parse(open(os.path.join(
    root, 'fluxvla/ops/triton/attention_triton_ops.py')).read())
direct = set()
for node in ast.walk(inf):
    if isinstance(node, ast.ImportFrom) and node.module == \
            'fluxvla.ops.triton.attention_triton_ops':
        direct |= {a.name for a in node.names}
for node in att.body:
    if isinstance(node, ast.FunctionDef) and node.name in direct:
        a = node.args
        names = [x.arg for x in a.args]
        defaults = [ast.literal_eval(d) for d in a.defaults]
        sigs['triton:' + node.name] = {
            'args': names,
            'defaults': dict(zip(names[len(names) - len(defaults):], defaults)),
            'line': node.lineno}
out = os.path.join(os.path.dirname(os.path.abspath(__file__)),
                   'atomic_ops_signatures.json')
with open(out, 'w') as f:
    json.dump(sigs, f, indent=1, sort_keys=True)
print(f'{len(sigs)} signatures -> {out}')
