"""Write topology files with the reference's own serializer, for interchange tests.

The reference package (``neurosim_gpu``) is imported from the checkout given by
``--reference`` (its ``src`` directory is put on ``sys.path``).  Two files of
``random_topology(300, 3000, seed=2)`` are written with the reference's
``save_topology`` (src/neurosim_gpu/topology_io.py:319-331): one plain, one with
the redundant destination weights.  tests/test_topology_io.py loads them with
this package's loader.

Run (only where the reference checkout exists):
    python tests/golden/make_topology_fixture.py --reference <path-to-reference-checkout>
The files are committed; nothing at test time reads the reference.
"""

from __future__ import annotations

import argparse
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--reference", required=True)
    args = parser.parse_args()
    sys.path.insert(0, str(Path(args.reference) / "src"))
    from neurosim_gpu.topology import random_topology
    from neurosim_gpu.topology_io import save_topology

    graph = random_topology(300, 3000, device="cpu", seed=2)
    save_topology(graph, HERE / "topology_ref_plain.pt")
    save_topology(graph, HERE / "topology_ref_with_in_weight.pt", include_destination_weights=True)
    print("wrote", HERE / "topology_ref_plain.pt", HERE / "topology_ref_with_in_weight.pt")


if __name__ == "__main__":
    main()
