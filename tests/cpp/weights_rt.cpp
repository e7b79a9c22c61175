// Round trip through the C++ host's .weights code (darknet_zig_b200/host/weights.hpp):
//   weights_rt IN OUT   loads IN into the test network of tests/test_weights.py, prints seen
//                       and each layer's first rolling_variance value (or "-"), saves OUT.
#include <cstdio>

#include "weights.hpp"

using dnb::weights::Kind;
using dnb::weights::Layer;

int main(int argc, char **argv) {
    if (argc != 3) {
        fprintf(stderr, "usage: %s IN OUT\n", argv[0]);
        return 2;
    }
    std::vector<Layer> net(4);
    net[0].kind = Kind::Convolutional, net[0].n = 8, net[0].batch_normalize = true, net[0].nweights = 8 * 4 * 3 * 3;
    net[1].kind = Kind::Connected, net[1].n = 5, net[1].batch_normalize = true, net[1].inputs = 12;
    net[2].kind = Kind::Batchnorm, net[2].n = 6;
    net[3].kind = Kind::Convolutional, net[3].n = 3, net[3].nweights = 3 * 8;
    for (Layer &l : net) l.allocate();
    try {
        const uint64_t seen = dnb::weights::load(argv[1], net);
        printf("seen %llu\n", (unsigned long long)seen);
        for (const Layer &l : net) {
            if (l.rolling_variance.empty())
                printf("-\n");
            else
                printf("%.9g\n", (double)l.rolling_variance[0]);
        }
        dnb::weights::save(argv[2], net, seen);
    } catch (const std::exception &e) {
        fprintf(stderr, "%s\n", e.what());
        return 1;
    }
    return 0;
}
