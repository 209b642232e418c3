/* TEST INFRASTRUCTURE ONLY: adapter for the unmodified reference build of
 * pickle_e2e.c. The reference's own attention block runs; nothing to attach. */
#include "pickle.h"
#include "pickle_fast.h"

int  e2e_attach(pickle_fast_state_t* st) { (void)st; return PICKLE_OK; }
void e2e_detach(void) {}
