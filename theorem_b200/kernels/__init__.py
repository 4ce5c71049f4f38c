"""Drop-in replacements for the reference's ``kernels/<op>/kernel.py`` modules.

Each subpackage exposes the same public names as the reference's
``kernel.py`` (``custom_kernel`` plus the launch-config tables the tooling
imports). ``ref_kernel`` / ``generate_input`` stay in the reference's own
``reference.py``; this package does not ship them.
"""
