"""The parity rules of the tests (defined with the oracle in ``oracle/parity.py``,
where ``bench.py``'s result check also reads them)."""
from oracle.parity import REL, REL_WEIGHTED, check_parity, check_rows_parity  # noqa: F401
