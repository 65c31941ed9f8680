"""Release and reproduction tooling: claim lines and the claims gate, recomputation of claims from evaluation
records, the hash-chained pre-registration ledger, tree manifests, field stripping of result trees and the secret /
privacy scan (the roles of recompute/gate.py, recompute/common.py and tools/*.py in the reference)."""
