"""CPU oracle for the GDN path -- test infrastructure only (see gdn_oracle.py)."""
