"""Regenerates tests/golden/topology_ref_hashes.json from the reference's own
Stage 2e topology generator (stage2e::init_synapses_host,
src/stage2e/network_init.cu:158-473), compiled unmodified from the reference
tree into oracle/_ref/topo_pin by oracle/ref/Makefile.  Run on the machine that
has the reference tree:

    make -C oracle/ref REF=<reference project>/src
    python tests/golden/make_topology_pin.py
"""
import json
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))

out = subprocess.run([os.path.join(ROOT, "oracle", "_ref", "topo_pin")], check=True,
                     capture_output=True, text=True).stdout
d = {}
for line in out.splitlines():
    k, _, v = line.partition(" ")
    if k == "sample":
        d[k] = v.split()
    elif k == "n_synapses":
        d[k] = int(v)
    else:
        d[k] = v.strip()
d["source"] = "reference src/stage2e/network_init.cu:158-473 via oracle/_ref/topo_pin"
with open(os.path.join(HERE, "topology_ref_hashes.json"), "w") as f:
    json.dump(d, f, indent=1)
print(json.dumps(d, indent=1))
