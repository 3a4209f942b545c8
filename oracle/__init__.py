"""CPU oracle for the int8 / int8-dyn quantised-linear path.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU-baseline leg may import this package, and only as the
checker (or, for the baseline, as the timed CPU restatement).  The product
package never imports it and has no CPU fallback.

``quant_ref``  numpy + C restatement of spikingbrain_cpu/quant.py (the checker).
``cpu_port``   a torch-CPU port of the reference forward passes, timed as the
               CPU baseline on the GPU host (the reference itself is not there).
"""
