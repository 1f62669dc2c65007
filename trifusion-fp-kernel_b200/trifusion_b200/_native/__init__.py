"""Holds the in-tree build of libtrifusion_b200.so (see ../../build.py)."""
