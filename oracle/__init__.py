"""CPU oracle for the KDA core (test infrastructure; see ``kda_oracle``)."""
