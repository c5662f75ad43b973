"""Caller-side restatement of Sheaf's lowering (ANF, reverse-mode AD,
simplify, StableHLO emission) and the benchmark programs built with it.

Test and benchmark infrastructure: it produces the StableHLO text that
Sheaf's JIT hands to the runtime, because Sheaf itself (Rust) cannot run
here.  The backend (`sheaf_b200`) never imports it.
"""
