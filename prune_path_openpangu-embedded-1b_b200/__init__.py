"""B200-native (sm_100a) PrunePath sparse-MoE MLP.

Import with ``importlib.import_module("prune_path_openpangu-embedded-1b_b200")`` (the
directory name is not a Python identifier).  Public API:

* ``TauSparseMoE`` -- drop-in for the reference's Triton module of the same name;
* ``IntegratedOpenPanguMoEMLP``, ``physical_reorder_for_inference`` -- caller-side mirrors;
* ``synth`` -- seeded synthetic layers and activations;
* ``ingest`` -- checkpoint state_dict + cluster files -> ``TauSparseMoE`` layers;
* ``training`` -- training-mode router outputs (softmax probabilities) and auxiliary losses;
* ``_lib`` -- the ctypes binding of ``libppmoe.so`` (C ABI in ``include/ppmoe.h``).
"""
from . import _lib, synth  # noqa: F401  (neither needs a GPU to import)


def __getattr__(name):
    if name in ("TauSparseMoE", "IntegratedOpenPanguMoEMLP", "physical_reorder_for_inference"):
        from . import tau_moe
        return getattr(tau_moe, name)
    if name in ("ingest", "training", "ep", "decoder"):
        import importlib
        return importlib.import_module(__name__ + "." + name)
    raise AttributeError(name)
