"""CPU oracle of the streaming semi-CRF scan (test infrastructure only)."""
