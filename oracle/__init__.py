"""CPU oracle of the KaniTTS decode-path kernels (test infrastructure only).

Imported by the tests, ``__graft_entry__.smoke()`` and the CPU-baseline leg
of ``bench.py`` as the checker; the product never imports it.
"""
