"""CPU oracle (test infrastructure): numpy restatements of the reference's
ALPHABET forward path and pole-residue Laplace layer, used only as the
parity checker by the tests, ``__graft_entry__.smoke()`` and ``bench.py``'s
CPU baseline."""
