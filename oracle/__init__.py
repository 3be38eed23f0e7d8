"""CPU oracle for the tensor-op hot path -- TEST INFRASTRUCTURE ONLY.

Imported only by tests/, __graft_entry__.smoke() and bench.py's CPU legs
(the cpu_baseline sample and the `--impl reference` arm).  The product
package never imports, links or falls back to anything here.
"""
