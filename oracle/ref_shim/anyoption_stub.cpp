// Link-time stand-ins for the two external dependencies of the reference's
// CPU drivers, so their compute templates can be built into oracle/_ref:
//   * AnyOption: a git submodule whose .cpp is absent from the reference
//     checkout; only its header (anyoption.h) is present.  The drivers'
//     main() functions use it; those are renamed and never called here.
//   * OpenBLAS cblas_* comparison calls, never reached from the oracle path.
// Every definition is a no-op.
#include "anyoption.h"
#include "cblas.h"

AnyOption::AnyOption() {}
AnyOption::~AnyOption() {}
void AnyOption::setOption(const char*) {}
void AnyOption::setOption(char) {}
void AnyOption::setOption(const char*, char) {}
void AnyOption::setFlag(const char*) {}
void AnyOption::setFlag(char) {}
void AnyOption::setFlag(const char*, char) {}
void AnyOption::processCommandArgs(int, char**) {}
char* AnyOption::getValue(const char*) { return nullptr; }
bool AnyOption::getFlag(const char*) { return false; }
char* AnyOption::getValue(char) { return nullptr; }
bool AnyOption::getFlag(char) { return false; }
void AnyOption::printUsage() {}
void AnyOption::addUsage(const char*) {}

extern "C" {
void cblas_sgemm(enum CBLAS_ORDER, enum CBLAS_TRANSPOSE, enum CBLAS_TRANSPOSE, int, int, int,
                 float, const float*, int, const float*, int, float, float*, int) {}
void cblas_ssymm(enum CBLAS_ORDER, enum CBLAS_SIDE, enum CBLAS_UPLO, int, int, float,
                 const float*, int, const float*, int, float, float*, int) {}
void cblas_sscal(int, float, float*, int) {}
void openblas_set_num_threads(int) {}
}
