"""Import helper: the package directory is named ``adapter-os_b200`` (not a
Python identifier), so tests load it through importlib."""
import importlib
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

aos = importlib.import_module("adapter-os_b200")
