"""Test infrastructure: CPU restatement of the reference's forward pass (the checker).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm may import this
package. The product (tiktoktechjam2026track3_b200) never does.
"""
