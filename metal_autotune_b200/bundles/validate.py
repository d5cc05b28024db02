"""`python -m metal_autotune_b200.bundles.validate <bundle_dir>`: see artifact.py."""
import sys

from .artifact import _main

if __name__ == "__main__":
    sys.exit(_main("validate"))
