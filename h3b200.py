"""Import shim: the package lives in the directory ``minimaxh3_on_k100-ai_b200``
(not a Python identifier); ``import h3b200`` loads it under this name."""
import importlib.util
import os
import sys

_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "minimaxh3_on_k100-ai_b200")
_spec = importlib.util.spec_from_file_location(__name__, os.path.join(_DIR, "__init__.py"),
                                               submodule_search_locations=[_DIR])
_module = importlib.util.module_from_spec(_spec)
sys.modules[__name__] = _module
_spec.loader.exec_module(_module)
