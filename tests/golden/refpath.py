"""Location of the reference source tree for the fixture generators: the
directory named by $ORCHKV_REFERENCE, else a `reference` checkout beside this
repository.  None when neither exists (the generators then stop with a
message; the committed fixtures do not need it)."""
import os

_REPO = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def reference_root():
    root = os.environ.get("ORCHKV_REFERENCE") or os.path.join(os.path.dirname(_REPO), "reference")
    return root if os.path.isdir(os.path.join(root, "python", "orchkv")) else None


def reference_file(rel):
    """Path of `rel` inside the reference tree (raises SystemExit if absent)."""
    root = reference_root()
    if root is None:
        raise SystemExit("reference tree not found: set ORCHKV_REFERENCE")
    return os.path.join(root, rel)
