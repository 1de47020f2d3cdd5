"""Interface shim of the Emmy 0.3.11 modules the reference compiler imports.

TEST INFRASTRUCTURE ONLY: it exists so that the reference's own compiler
(``ptx_backend.compile_file`` of the Lazy-Compiler checkout) can run
unchanged in this container and print the PTX it would emit.  It is written
from the way the reference uses Emmy (isinstance dispatch, node attributes,
``defines`` / ``deps`` / ``exprs`` / ``free_vars`` queries, accumulator
identities, ``Dim.as_static``, ``Graph.from_dict``), not from Emmy's
sources, which are not available here.  Fidelity is checked by the SHA-256
of the emitted PTX against the hashes the reference recorded for the same
IR files (``oracle/ref_ptx.py``).
"""
