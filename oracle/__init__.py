"""CPU oracle for the block-quantized hot path (test infrastructure only).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this
package.  The product library never imports it.
"""
