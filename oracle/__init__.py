"""Oracle package: CPU restatement of the reference PGF algorithm.  Test infrastructure only."""
