"""CPU oracle package: test infrastructure only (see emul_oracle.c).  Never imported by the product."""
