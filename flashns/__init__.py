"""The reference's import name for the evaluation path.

``import flashns`` and ``from flashns.pinn_packed import PackedPINN`` resolve to this
library's modules, so code written against the reference's ``flashns`` package
(``src/flashns/``) runs on the B200 kernels without edits to its imports.

Only the six modules of the evaluation path are provided: ``jet_spec``, ``jet_stable``,
``jet_packed``, ``ns_seed``, ``pinn_packed`` and ``distributed_contract``.  Each is the
``flashns_b200`` module object itself (``flashns.pinn_packed is flashns_b200.pinn_packed``),
not a copy.  The reference's other modules (Euler and spline solvers, CLI, provenance,
diagnostics) lie outside this path and are not provided.
"""

import importlib
import sys

MODULES = ("jet_spec", "jet_stable", "jet_packed", "ns_seed", "pinn_packed", "distributed_contract")

for _name in MODULES:
    _module = importlib.import_module(f"flashns_b200.{_name}")
    sys.modules[f"{__name__}.{_name}"] = _module
    globals()[_name] = _module
del _name, _module
