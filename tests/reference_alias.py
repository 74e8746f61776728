"""pytest plugin: makes ``mini_infra.core`` (the reference's control-plane package) resolve to
``mini_infra_b200.core``, so that the reference's own control-plane unit tests run unchanged
against this package (``tests/test_reference_control_plane.py`` loads it with ``-p``)."""

import sys
import types

import mini_infra_b200.core as core

_pkg = types.ModuleType("mini_infra")
_pkg.__path__ = []  # a namespace with only the aliased sub-module
_pkg.core = core
sys.modules["mini_infra"] = _pkg
sys.modules["mini_infra.core"] = core
