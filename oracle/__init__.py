"""CPU oracle of the Kitty hot path - TEST INFRASTRUCTURE ONLY.

Imported only by ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline
leg of ``bench.py`` as the checker / the timed CPU restatement; the ``kitty``
package never imports it.  See ``kitty_oracle.py`` for the function-by-function
correspondence with the reference (bitxwolf/kitty-kv).
"""
