"""ORACLE - test infrastructure only: CPU restatements used to check the CUDA library.

Only ``tests/``, ``__graft_entry__.smoke`` and the CPU-baseline leg of ``bench.py`` import this
package; the product (``pov-shuffle_b200/povs``) never does.
"""
