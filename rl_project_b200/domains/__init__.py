"""Application domains built on the framework: pharmaceutical synthesis and budgeted allocation."""
