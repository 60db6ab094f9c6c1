// Library-wide C entry points (version, error string).
#include "../../include/genie_tk_b200.h"
#include "gtk_host.h"

extern "C" {

int gtk_version(void) { return 100; }  // 0.1.0

const char* gtk_last_error_string(void) { return gtk::last_error(); }

}  // extern "C"
