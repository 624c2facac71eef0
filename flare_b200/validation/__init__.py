"""Validation tools over this framework's traces, audits and placements (see the submodules)."""
